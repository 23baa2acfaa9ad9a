"""Decode benchmark: batched greedy KV-cache decoding with segment-tree attention.

Model: 12 layers, d_model 768, 12 heads (dh 64), vocab 50304, random init N(0, 0.02), bf16 weights and cache.
Input: batch 64 prompts of 4096 uniform-random tokens per GPU (seeded per rank), prefilled untimed, then greedy
decode steps; tree: 64-token leaves, top-16 leaves, 128-token local window, Tcap 8192.

One step = one greedy decode step of the whole batch through all 12 layers + lm_head (CUDA graph).
  value    tokens/s over all ranks, device-resident loop (tokens fed back on the device)
  e2e      tokens/s through Decoder.serve_step: tokens copied host->device from pinned memory and the next tokens
           device->host every step
  roofline the fused decode-attention kernel (ta_decode_step) timed alone with CUDA events: selected-KV bytes per
           launch / launch time vs the measured HBM copy bandwidth
  strong   (under torchrun) the same 64 sequences split over the ranks, 64 / N each: tokens/s, speed-up and
           efficiency against this run's own 1-GPU step time
  kernels  (N=1) configurations 1, 2, 3 and 5: the whole configuration-1 forward, the configuration-2 gather-dot,
           one configuration-3 prefill attention layer and the configuration-5 decode kernel, each against its
           roofline with its own clock record
Multi-GPU: one process per GPU (torchrun), each rank decodes its own 64 sequences; no collective in the timed
region (weak scaling). `--impl reference` times the CPU oracle (numpy restatement of the reference's engine) on
the host cores instead.
"""
import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)


class Spec:
    """A decode-engine configuration of BASELINE.json (model, tree and run)."""

    def __init__(self, name, V, C, H, NL, leaf, topk, window, tcap, batch, prompt, fill):
        self.name, self.V, self.C, self.H, self.NL = name, V, C, H, NL
        self.leaf, self.topk, self.window, self.tcap = leaf, topk, window, tcap
        self.batch, self.prompt, self.fill = batch, prompt, fill
        self.dh = C // H


# configuration 4: prompts run through the model (prefill), then greedy decoding
CFG4 = Spec('4', V=50304, C=768, H=12, NL=12, leaf=64, topk=16, window=128, tcap=8192, batch=64, prompt=4096,
            fill='prefill')
# configuration 5: 32768-token contexts; the caches are filled with random keys/values (the decode cost does not
# depend on their values) and the trees built from them, since a 24-layer prefill of the contexts is not the
# measured step; batch per GPU is what fits in HBM (256 sequences need 1.65 TB of KV: more than 8 GPUs hold)
CFG5 = Spec('5', V=32000, C=2048, H=16, NL=24, leaf=128, topk=32, window=256, tcap=65536, batch=20, prompt=32768,
            fill='random')
V, C, H, NL = CFG4.V, CFG4.C, CFG4.H, CFG4.NL
LEAF, TOPK, WINDOW, TCAP = CFG4.leaf, CFG4.topk, CFG4.window, CFG4.tcap
# own kernels per greedy step: embed+LN; per layer the fused decode attention, 2 x add+LN and GELU; argmax+advance
# (the projections are cuBLAS)
METRIC = 'decode tok/s (config 4: 12x768 bf16 GPT, batch 64/GPU, 4096-token prompts, leaf 64, top-16, window 128)'
METRIC5 = 'decode tok/s (config 5: 24x2048 bf16 GPT, 32768-token contexts, leaf 128, top-32, window 256)'


def parse():
    p = argparse.ArgumentParser()
    p.add_argument('--gpus', type=int, default=1)
    p.add_argument('--steps', type=int, default=256)
    p.add_argument('--warmup', type=int, default=8)
    p.add_argument('--impl', default='ours', choices=['ours', 'reference'])
    p.add_argument('--batch', type=int, default=64)
    p.add_argument('--prompt', type=int, default=4096)
    p.add_argument('--no-cpu-baseline', action='store_true')
    p.add_argument('--cpu-seconds', type=float, default=12.0)
    p.add_argument('--splits', type=int, default=0, help='CTAs per (b, h) in the decode kernel (0 = auto)')
    p.add_argument('--config5', action='store_true',
                   help='configuration 5 instead of 4: 24 layers x 2048 (16 heads, dh 128, vocab 32000), 128-token '
                        'leaves, top-32, window 256, 32768-token contexts (random-filled caches), 128 steps, 20 '
                        'sequences per GPU (what fits in HBM); with --kernel-only the decode kernel alone at '
                        'batch 32')
    p.add_argument('--kernel-only', action='store_true',
                   help='time only the fused decode kernel on the config-4 shape (random caches of 4 layers, '
                        'rotated so that no launch finds its KV in L2) and print one JSON line')
    p.add_argument('--gather-dot', action='store_true',
                   help='configuration 2 instead: the block gather-dot kernel alone (B=8, H=12, dh=64, T=4096 bf16, '
                        '16 sorted unique 64-token blocks per (b, h)); prints one JSON line')
    p.add_argument('--prefill-attn', action='store_true',
                   help='configuration 3 instead: one layer of prefill sparse attention (B=4, H=12, T=8192, dh=64 '
                        'bf16, leaf 64, top-16, window 128; selection from the tree kernels on random q/k), timing the '
                        'tensor-core tile kernel and the warp-per-query kernel; prints one JSON line')
    p.add_argument('--config1', action='store_true',
                   help='configuration 1 instead: the full forward of the 4-layer d=256 fp32 GPT (B=2, T=512, leaf 32, '
                        'top-4, window 64) on the GPU and on the CPU oracle, logits compared; prints one JSON line')
    p.add_argument('--block', action='store_true',
                   help="the block forest's TreeAttention (attn='block') at train.py's and a 4096-token configuration; "
                        'prints one JSON line each')
    p.add_argument('--dyn', action='store_true',
                   help="the dynamic content tree's select_keys (attn='dyn') at train.py's and a 4096-token "
                        'configuration; prints one JSON line each')
    p.add_argument('--config3', action='store_true',
                   help='configuration 3 end to end: the 12-layer bf16 GPT forward (prefill) over 4 x 8192 tokens; '
                        'prints one JSON line')
    p.add_argument('--fused-linear', type=int, default=-1,
                   help='1: the decode step\'s projections on the library\'s tensor-core kernel where Decoder.lin_splits '
                        'says so (ta_linear_rows, K-split c_proj / c_mlp); 0: every projection on cuBLAS; -1 (default): '
                        'the Decoder\'s choice (the library kernel for batches of at most 32 sequences)')
    p.add_argument('--no-kernels', action='store_true',
                   help='default run: skip the kernels sub-record (configurations 1, 2, 3 and 5 measured after the '
                        'decode loop)')
    p.add_argument('--no-strong', action='store_true',
                   help='default run under torchrun: skip the fixed-global-batch (strong scaling) decode loop')
    p.add_argument('--profile-steps', type=int, default=0,
                   help='profiling mode: after prefill and warm-up run this many eager decode steps between '
                        'cudaProfilerStart/Stop (for ncu --profile-from-start off) and exit')
    return p.parse_args()


def make_cfg(M):
    from treeattn_b200.config import Config
    return Config(vocab_size=M.V, seq_len=M.tcap, n_layer=M.NL, n_head=M.H, n_embd=M.C, attn='seg', wmax=M.topk,
                  beam=M.topk, local=M.window, neighbors=False, beam_mode='fixed', leaf=M.leaf)


def make_weights(device, seed, dtype, M=CFG4):
    """Random-init weights of the architecture (GPT._init: N(0, 0.02), c_proj 0.02/sqrt(2L))."""
    g = torch.Generator(device=device).manual_seed(seed)
    n = lambda *s, std=0.02: (torch.randn(*s, generator=g, device=device) * std).to(dtype)
    sp = 0.02 / math.sqrt(2 * M.NL)
    C = M.C
    W = dict(wte=n(M.V, C), wpe=n(M.tcap, C), ln_f=torch.ones(C, device=device), layers=[])
    for _ in range(M.NL):
        W['layers'].append(dict(ln1=torch.ones(C, device=device), c_attn=n(3 * C, C), c_proj=n(C, C, std=sp),
                                ln2=torch.ones(C, device=device), c_fc=n(4 * C, C), c_mlp=n(C, 4 * C, std=sp)))
    return W


class Clocks:
    """nvidia-smi sampling of SM clocks and throttle reasons; only samples inside [t_begin, t_end] are kept."""
    Q = ('timestamp,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,'
         'clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,'
         'clocks_event_reasons.sw_power_cap')

    def __init__(self, index):
        self.index, self.proc, self.path = index, None, None
        self.t_begin = self.t_end = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix='.csv')
            os.close(fd)
            self.proc = subprocess.Popen(['nvidia-smi', '-i', str(self.index), '--query-gpu=' + self.Q,
                                          '--format=csv,noheader,nounits', '-lms', '50'],
                                         stdout=open(self.path, 'w'), stderr=subprocess.DEVNULL)
            time.sleep(1.0)  # let the sampler come up before the timed region
        except Exception:
            self.proc = None

    def mark_begin(self):
        self.t_begin = time.time()

    def mark_end(self):
        self.t_end = time.time()

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.1)
        self.proc.terminate()
        try:
            self.proc.wait(5)
        except Exception:
            self.proc.kill()
        from datetime import datetime
        rows = []
        for line in open(self.path):
            f = [x.strip() for x in line.split(',')]
            if len(f) < 9:
                continue
            try:
                ts = datetime.strptime(f[0], '%Y/%m/%d %H:%M:%S.%f').timestamp()
            except ValueError:
                continue
            if self.t_begin - 0.05 <= ts <= self.t_end + 0.05:
                rows.append(f)
        os.unlink(self.path)
        if not rows:
            return dict(sm_mhz=None, sm_max_mhz=None, reasons=[], samples=0)
        num = lambda x: float(x) if x.replace('.', '', 1).isdigit() else None
        sm = [v for v in (num(r[1]) for r in rows) if v is not None]
        smax = [v for v in (num(r[2]) for r in rows) if v is not None]
        names = ['hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown', 'sw_power_cap']
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i] == 'Active'})
        return dict(sm_mhz=statistics.median(sm) if sm else None, sm_max_mhz=max(smax) if smax else None,
                    reasons=reasons, samples=len(rows))


def profiled_traffic():
    """DRAM bytes (read + write) per launch of the decode kernel from the committed ncu summary, or None."""
    try:
        for line in open(os.path.join(ROOT, 'profiles', 'decode_kernel_config4.md')):
            if line.startswith('traffic_bytes_per_launch:'):
                return float(line.split(':')[1])
    except OSError:
        pass
    return None


def measured_peaks():
    try:
        return json.load(open(os.path.join(ROOT, 'MEASURED_PEAKS.json')))
    except Exception:
        return None


def _cpu_decoder_rate(M, seconds, W, n_layers, seed):
    """Steps per second of the CPU oracle's decoder (batch 1) with n_layers layers, prompt cache of M.prompt
    random positions per layer."""
    import numpy as np

    import oracle
    rng = np.random.default_rng(seed)
    W = dict(W, layers=W['layers'][:n_layers])
    T0 = M.prompt
    dec = oracle.DecoderNP(W, M.H, M.tcap, M.topk, M.topk, M.window, L0=int(math.log2(M.leaf)), cap=T0 + 512)
    dec.reset(1)
    for st in dec.states[0]:
        st.fill(rng.standard_normal((M.H, T0, M.dh), dtype=np.float32),
                rng.standard_normal((M.H, T0, M.dh), dtype=np.float32))
    tok = rng.integers(0, M.V, 1)
    dec.step(tok, T0)  # warm-up
    t0 = time.perf_counter()
    steps = 0
    while True:
        logits, _ = dec.step(tok, T0 + 1 + steps)
        tok = logits.argmax(-1)
        steps += 1
        if time.perf_counter() - t0 > seconds or steps >= 512:
            break
    return steps / (time.perf_counter() - t0), steps


def cpu_decode_sample(seconds, W_dev=None, seed=0, M=CFG4):
    """Time the CPU oracle's decode (numpy, fp32, the reference engine's algorithm: engine.py:149-177 Decoder,
    batch 1) for a bounded number of steps. The prompt caches are filled with random keys/values instead of a CPU
    prefill (the time of a decode step does not depend on the values). Configuration 4 runs the whole model;
    for larger models (configuration 5: 24 layers, 32768-token caches) one- and two-layer decoders are timed and
    the step is extrapolated to all layers (t1 + (NL - 1) (t2 - t1)). Returns (tokens/s, steps, threads, how)."""
    import numpy as np
    rng = np.random.default_rng(seed)
    if W_dev is not None:
        f = lambda t: t.float().cpu().numpy()
        W = dict(wte=f(W_dev['wte']), wpe=f(W_dev['wpe']), ln_f=f(W_dev['ln_f']),
                 layers=[{k: f(v) for k, v in L.items()} for L in W_dev['layers']])
    else:
        n = lambda *s, std=0.02: (rng.standard_normal(s, dtype=np.float32) * std)
        C = M.C
        nl = M.NL if M is CFG4 else 2
        W = dict(wte=n(M.V, C), wpe=n(M.tcap, C), ln_f=np.ones(C, np.float32),
                 layers=[dict(ln1=np.ones(C, np.float32), c_attn=n(3 * C, C), c_proj=n(C, C),
                              ln2=np.ones(C, np.float32), c_fc=n(4 * C, C), c_mlp=n(C, 4 * C)) for _ in range(nl)])
    if M is CFG4:
        rate, steps = _cpu_decoder_rate(M, seconds, W, M.NL, seed)
        return rate, steps, _cpu_threads(), '%d greedy decode steps of 1 sequence at t~%d' % (steps, M.prompt)
    r1, s1 = _cpu_decoder_rate(M, seconds / 2, W, 1, seed)
    r2, s2 = _cpu_decoder_rate(M, seconds / 2, W, 2, seed)
    t1, t2 = 1.0 / r1, 1.0 / r2
    t_step = t1 + (M.NL - 1) * max(t2 - t1, 0.0)
    return 1.0 / t_step, s1 + s2, _cpu_threads(), (
        '%d + %d greedy steps of 1 sequence at t~%d with 1- and 2-layer decoders (%.1f / %.1f ms), extrapolated to '
        '%d layers' % (s1, s2, M.prompt, t1 * 1e3, t2 * 1e3, M.NL))


def _cpu_threads():
    try:
        from threadpoolctl import threadpool_info
        return max([i.get('num_threads', 1) for i in threadpool_info()] + [1])
    except Exception:
        return 1


def cpu_gather_dot_sample(q, K, blocks, blk, byts, seconds=4.0):
    """Configuration 2 on the host: the CPU oracle's gather_dot (the reference's torch fallback form,
    fastseg.py:121-122) on the same q, K and block ids, repeated for a bounded time; GB/s on the same
    algorithmic bytes as the kernel."""
    import numpy as np

    import oracle
    qn = q.float().cpu().numpy()[:, :, None]
    Kn = K.float().cpu().numpy()
    bl = blocks.long().cpu().numpy()
    cand = (bl[..., None] * blk + np.arange(blk)).reshape(bl.shape[0], bl.shape[1], 1, -1)
    oracle.gather_dot(qn, Kn, cand, 0.125)
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        oracle.gather_dot(qn, Kn, cand, 0.125)
        n += 1
    dt = (time.perf_counter() - t0) / n
    return dict(value=byts / dt / 1e9, unit='GB/s', cores=_cpu_threads(), kind='port',
                sample='%d calls of the full configuration-2 gather-dot (numpy fp32 oracle), %.2f ms each' % (n, dt * 1e3))


def cpu_prefill_sample(q, k, v, leaf, topk, window):
    """Configuration 3 on the host: the CPU oracle's SegAttention.sparse_attend (fastseg.py:345-389: levels,
    descent, static keys, dedupe, exact attention) for ONE (b, h) of the whole 8192-token sequence, fp32 numpy;
    TFLOP/s on that head's algorithmic FLOPs (4 dh per kept key per query)."""
    import numpy as np

    import oracle
    qh, kh, vh = [t[:1, :1].float().cpu().numpy() for t in (q, k, v)]
    t0 = time.perf_counter()
    _, stats = oracle.seg_attention(qh, kh, vh, topk, topk, window, L0=int(math.log2(leaf)))
    dt = time.perf_counter() - t0
    flops = 4.0 * qh.shape[-1] * stats['keys_total'] * qh.shape[2]
    return dict(value=flops / dt / 1e12, unit='TFLOP/s', cores=_cpu_threads(), kind='port',
                sample='one (b, h) of 8192 queries (selection + attention, numpy fp32 oracle) in %.2f s; the GPU '
                       'figure covers 48 (b, h)' % dt)


def run_kernel_only(a, dev, emit=True):
    """Config-4 decode-attention kernel alone: batch a.batch x 12 heads, dh 64, bf16 caches holding a.prompt
    positions, leaf 64, top-16, window 128, position t = prompt (+ the launch index). With --profile-steps the
    launches are bracketed by cudaProfilerStart/Stop for ncu."""
    from treeattn_b200 import _ops
    from treeattn_b200._ops import Levels
    if a.config5:
        Hh, dh, leaf, topk, window, tcap = 16, 128, 128, 32, 256, 65536
        B, T0 = a.batch if a.batch != 64 else 32, (32768 if a.prompt == 4096 else a.prompt)
    else:
        Hh, dh, leaf, topk, window, tcap = H, C // H, LEAF, TOPK, WINDOW, TCAP
        B, T0 = a.batch, a.prompt
    Cm = Hh * dh
    L0, Lm = int(math.log2(leaf)), int(math.log2(tcap)) - 1
    cap = T0 + 64
    nlay = 1 if a.profile_steps else 4  # profiling: one layer's caches (ncu restores device memory per pass)
    g = torch.Generator(device=dev).manual_seed(7)
    layers = []
    for _ in range(nlay):
        K = (torch.randn(B, Hh, cap, dh, device=dev, generator=g) * 0.5).to(torch.bfloat16)
        Vv = torch.randn(B, Hh, cap, dh, device=dev, generator=g).to(torch.bfloat16)
        lv = Levels.empty(B, Hh, dh, cap, L0, Lm, dev)
        _ops.build_levels(K[:, :, :T0], cap, L0, Lm, zero_sink=True, out=lv)
        layers.append((K, Vv, lv))
    qkv = torch.randn(B, 3 * Cm, device=dev, generator=g).to(torch.bfloat16)
    pos = torch.full((B,), T0, device=dev, dtype=torch.int32)
    att = torch.empty(B, Cm, device=dev, dtype=torch.bfloat16)
    nk = torch.empty(B, Hh, device=dev, dtype=torch.int32)
    splits = a.splits or _ops.default_splits(B, Hh, dh, torch.bfloat16)
    scratch = _ops.split_scratch(B, Hh, dh, dev)

    def run_all():
        for K, Vv, lv in layers:
            _ops.decode_step(qkv, K, Vv, lv, pos, Hh, topk, topk, window, 1 / math.sqrt(dh), att, nkeys=nk,
                             splits=splits, scratch=scratch)

    run_all()
    torch.cuda.synchronize()
    if a.profile_steps:
        torch.cuda.cudart().cudaProfilerStart()
        for _ in range(a.profile_steps):
            run_all()
        torch.cuda.synchronize()
        torch.cuda.cudart().cudaProfilerStop()
        print(json.dumps(dict(kernel_only=True, profile_steps=a.profile_steps, launches=nlay * a.profile_steps)))
        return
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s), torch.cuda.graph(gr, stream=s):
        run_all()
    torch.cuda.current_stream(dev).wait_stream(s)
    gr.replay()
    torch.cuda.synchronize()
    reps = 25
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        gr.replay()
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / (reps * nlay)
    byts = float(nk.sum()) * dh * 2 * 2
    peaks = measured_peaks()
    peak = peaks['hbm_gbs'] if peaks else 6650.0
    line = dict(kernel_only=True, config='5' if a.config5 else '4', batch=B, heads=Hh, dh=dh, prompt=T0,
                splits=splits, kernel_us=us, bytes_per_launch=byts, achieved_gbs=byts / us / 1e3,
                frac=byts / us / 1e3 / peak, keys_per_head=float(nk.float().mean()))
    if emit:
        print(json.dumps(line), flush=True)
    return line


def run_gather_dot(a, dev, emit=True):
    """Configuration 2: per (b, h), scores of q against the 1024 keys of 16 selected 64-token blocks (fp32 out).
    The 13 MB working set fits in L2, so ROT independent copies of K (> L2 in total) are cycled through."""
    from treeattn_b200 import _ops
    B, H, T, dh, blk, nblk = 8, 12, 4096, 64, 64, 16
    ROT = 16
    g = torch.Generator(device=dev).manual_seed(3)
    Ks = [torch.randn(B, H, T, dh, device=dev, generator=g).to(torch.bfloat16) for _ in range(ROT)]
    q = torch.randn(B, H, dh, device=dev, generator=g).to(torch.bfloat16)
    blocks = torch.stack([torch.randperm(T // blk, device=dev, generator=g)[:nblk].sort().values
                          for _ in range(B * H)]).view(B, H, nblk).int()
    out = torch.empty(B, H, nblk * blk, device=dev, dtype=torch.float32)
    for K in Ks:
        _ops.gather_dot_blocks(q, K, blocks, blk, 0.125, nb_cta=1, out=out)
    torch.cuda.synchronize()
    if a.profile_steps:
        torch.cuda.cudart().cudaProfilerStart()
        for K in Ks[:a.profile_steps]:
            _ops.gather_dot_blocks(q, K, blocks, blk, 0.125, nb_cta=1, out=out)
        torch.cuda.synchronize()
        torch.cuda.cudart().cudaProfilerStop()
        return
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s), torch.cuda.graph(gr, stream=s):
        for K in Ks:
            _ops.gather_dot_blocks(q, K, blocks, blk, 0.125, nb_cta=1, out=out)
    torch.cuda.current_stream(dev).wait_stream(s)
    gr.replay()
    torch.cuda.synchronize()
    reps = 50
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        gr.replay()
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / (reps * ROT)
    byts = B * H * nblk * blk * dh * 2 + B * H * dh * 2 + B * H * nblk * 4 + B * H * nblk * blk * 4
    peaks = measured_peaks()
    peak = peaks['hbm_gbs'] if peaks else 6650.0
    line = dict(gather_dot=True, config='B=8 H=12 dh=64 T=4096 bf16, 16 blocks of 64 per (b,h)',
                kernel_us=us, bytes_per_call=byts, achieved_gbs=byts / us / 1e3, frac=byts / us / 1e3 / peak,
                rotated_copies=ROT)
    if not a.no_cpu_baseline:
        line['cpu_baseline'] = cpu_gather_dot_sample(q, Ks[0], blocks, blk, byts, seconds=min(a.cpu_seconds, 4.0))
    if emit:
        print(json.dumps(line), flush=True)
    return line


def union_tile_pairs(ids, vld, n_tree, leaf, Lw, T, qt=128, kt=64):
    """(query tile, key tile) pairs the prefill tile kernel streams: per (b, h, 128-query tile) the union of the
    used leaves' key tiles (parts before each query's window), the window tiles and tile 0."""
    B, H, N, wl = ids.shape
    dev = ids.device
    t = torch.arange(N, device=dev)
    w0 = (t - Lw + 1).clamp(min=0)
    slot = torch.arange(wl, device=dev)
    used = vld.bool() & (slot < n_tree) & (ids >= 0) & (ids * leaf < w0.view(1, 1, N, 1))
    ntq, ntk = -(-N // qt), -(-T // kt)
    occ = torch.zeros(B, H, ntq, ntk, dtype=torch.bool, device=dev)
    per = max(leaf // kt, 1)
    for j in range(per):  # key tiles a leaf spans (leaf >= kt) or the tile holding it (leaf < kt)
        tile = (ids.clamp(min=0) * leaf // kt + j).clamp(max=ntk - 1)
        qi = (t // qt).view(1, 1, N, 1).expand_as(tile)
        bi = torch.arange(B, device=dev).view(B, 1, 1, 1).expand_as(tile)
        hi = torch.arange(H, device=dev).view(1, H, 1, 1).expand_as(tile)
        occ[bi[used], hi[used], qi[used], tile[used]] = True
    for q0 in range(ntq):
        lo, hi_ = int(w0[q0 * qt]) // kt, min(q0 * qt + qt - 1, N - 1) // kt
        occ[:, :, q0, lo:hi_ + 1] = True
        if int(w0[min(q0 * qt + qt - 1, N - 1)]) > 0:
            occ[:, :, q0, 0] = True
    return int(occ.sum())


def run_block(a, dev):
    """The block forest's attention (attn='block', TreeAttention) at the reference's train.py configuration
    (B=8, 6 heads, 512 tokens, dh 64, 64-key blocks, wmax 8, beam 4) and a 4096-token window at B=2, bf16 q, k, v
    ~ N(0, 1): one layer's sparse_attend (build: ta_lane_order + ta_forest_levels; descent: ta_forest_select;
    attention: ta_sparse_attn) and the 6-layer GPT's forward, CUDA events after warm-up; the CPU oracle on one
    (b, h) as the baseline. Prints one JSON line per configuration."""
    from treeattn_b200.attention import TreeAttention
    from treeattn_b200.config import Config
    from treeattn_b200.forest import build_forest_raw
    from treeattn_b200.model import GPT
    ev = lambda: torch.cuda.Event(enable_timing=True)

    def timed(fn, reps=10):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        e0, e1 = ev(), ev()
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps

    for name, (B, H, T, dh, blk, wmax, beam) in dict(train=(8, 6, 512, 64, 64, 8, 4),
                                                     long=(2, 6, 4096, 64, 64, 8, 4)).items():
        cfg = Config(vocab_size=8192, seq_len=T, n_layer=6, n_head=H, n_embd=H * dh, attn='block', tree_block=blk,
                     wmax=wmax, beam=beam)
        g = torch.Generator(device=dev).manual_seed(13)
        q, k, v = [torch.randn(B, H, T, dh, device=dev, generator=g).to(torch.bfloat16) for _ in range(3)]
        m = TreeAttention(cfg).to(dev, torch.bfloat16).eval()
        if a.profile_steps:
            if name != 'long':
                continue
            with torch.no_grad():
                for _ in range(3):
                    m.sparse_attend(q, k, v)
                torch.cuda.synchronize()
                torch.cuda.cudart().cudaProfilerStart()
                for _ in range(a.profile_steps):
                    m.sparse_attend(q, k, v)
                torch.cuda.synchronize()
                torch.cuda.cudart().cudaProfilerStop()
            return
        with torch.no_grad():
            attn_ms = timed(lambda: m.sparse_attend(q, k, v))
            depth = int(round(math.log2(blk // 2)))
            build_ms = timed(lambda: build_forest_raw(k, blk, depth, cfg, zero_sink=True))
            model = GPT(cfg).to(dev, torch.bfloat16).eval()
            idx = torch.randint(0, cfg.vocab_size, (B, T), device=dev, generator=g)
            fwd_ms = timed(lambda: model(idx), reps=5)
        line = dict(block_attn=True, config='%s: B=%d H=%d T=%d dh=%d bf16, blocks of %d, wmax %d, beam %d' % (
            name, B, H, T, dh, blk, wmax, beam), layer_ms=attn_ms, build_ms=build_ms,
            queries_per_s=B * H * T / (attn_ms * 1e-3), gpt6_forward_ms=fwd_ms, gpt6_tokens_per_s=B * T / (fwd_ms * 1e-3),
            keys_per_query=float(m.aux['keys_total']))
        if not a.no_cpu_baseline:
            import oracle
            qn, kn, vn = [x[:1, :1].float().cpu().numpy() for x in (q, k, v)]
            t0 = time.perf_counter()
            oracle.tree_attention(qn, kn, vn, blk, wmax, beam)
            dt = time.perf_counter() - t0
            line['cpu_baseline'] = dict(value=T / dt, unit='queries/s', cores=1, kind='port',
                                        sample='oracle.tree_attention on one (b, h) of %d queries' % T)
        print(json.dumps(line), flush=True)


def run_dyn(a, dev):
    """The dynamic content tree's key selection (attn='dyn', dyntree.select_keys) at the reference's training
    configurations: train.py's defaults (B=8, 6 heads, 512 tokens, dh 64, lanes of 64, wmax 8, neighbours on) and a
    4096-token window (long_train.py's length) at B=2. q, k ~ N(0, 1) fp32, leaf budgets uniform in [2, wmax].
    CUDA events around whole select_keys calls (build: ta_lane_order + ta_lane_sums; loop: ta_lane_select) after
    warm-up; the CPU oracle (numpy) on one (b, h) as the baseline. Prints one JSON line per configuration."""
    from treeattn_b200 import dyntree
    from treeattn_b200.config import Config
    ev = lambda: torch.cuda.Event(enable_timing=True)
    for name, (B, H, T, dh, Y, wmax) in dict(train=(8, 6, 512, 64, 64, 8), long=(2, 6, 4096, 64, 64, 8)).items():
        cfg = Config(attn='dyn', seq_len=T, chunk=Y, wmax=wmax)
        g = torch.Generator(device=dev).manual_seed(11)
        q = torch.randn(B, H, T, dh, device=dev, generator=g)
        k = torch.randn(B, H, T, dh, device=dev, generator=g)
        lhat = torch.randint(2, wmax + 1, (B, H, T), device=dev, generator=g)
        nl = T // Y
        P = B * H * nl
        D = T.bit_length() - 2
        for _ in range(3):
            dyntree.select_keys(q, k, lhat, cfg)
        torch.cuda.synchronize()
        if a.profile_steps:
            if name != 'long':
                continue
            torch.cuda.cudart().cudaProfilerStart()
            for _ in range(a.profile_steps):
                dyntree.select_keys(q, k, lhat, cfg)
            torch.cuda.synchronize()
            torch.cuda.cudart().cudaProfilerStop()
            return
        reps = 5
        e0, e1 = ev(), ev()
        e0.record()
        for _ in range(reps):
            dyntree.select_keys(q, k, lhat, cfg)
        e1.record()
        torch.cuda.synchronize()
        total_ms = e0.elapsed_time(e1) / reps
        # the build alone
        n0 = (torch.arange(nl, device=dev, dtype=torch.int64) * Y).repeat(B * H)
        e0.record()
        for _ in range(reps):
            dyntree._order(k, nl, n0, 1, P, T, dh, cfg.kmeans_iters, D)
        e1.record()
        torch.cuda.synchronize()
        order_ms = e0.elapsed_time(e1) / reps
        line = dict(dyn_select=True, config='%s: B=%d H=%d T=%d dh=%d lanes of %d, wmax %d, neighbours on' % (
            name, B, H, T, dh, Y, wmax), lanes=P, select_keys_ms=total_ms, order_ms=order_ms,
            queries_per_s=B * H * T / (total_ms * 1e-3))
        if not a.no_cpu_baseline:
            import oracle
            qn, kn, ln = q[:1, :1].cpu().numpy(), k[:1, :1].cpu().numpy(), lhat[:1, :1].cpu().numpy()
            t0 = time.perf_counter()
            oracle.select_keys(qn, kn, ln, Y, wmax, cfg.nb_window, cfg.nb_store, cfg.nb_rho, cfg.nb_probe,
                               cfg.nb_cap_min)
            dt = time.perf_counter() - t0
            line['cpu_baseline'] = dict(value=T / dt, unit='queries/s', cores=1, kind='port',
                                        sample='oracle.select_keys on one (b, h) of %d queries' % T)
        print(json.dumps(line), flush=True)


def run_config3(a, dev):
    """Configuration 3 end to end: the whole 12-layer, 768-wide bf16 GPT forward (SegAttention prefill: levels,
    tile select, tensor-core tile attention; cuBLAS projections) over B=4 sequences of 8192 uniform-random tokens,
    leaf 64, top-16, window 128; CUDA events over whole forwards (inputs far above L2). Prints one JSON line."""
    from treeattn_b200.config import Config
    from treeattn_b200.model import GPT
    B = a.batch if a.batch != 64 else 4
    T = 8192
    cfg = Config(vocab_size=50304, seq_len=T, n_layer=12, n_head=12, n_embd=768, attn='seg', wmax=16, beam=16,
                 local=128, neighbors=False, beam_mode='fixed', leaf=64)
    torch.manual_seed(0)
    m = GPT(cfg).eval().to(dev, torch.bfloat16)
    idx = torch.randint(0, cfg.vocab_size, (B, T), device=dev, generator=torch.Generator(device=dev).manual_seed(5))
    ev = lambda: torch.cuda.Event(enable_timing=True)
    with torch.no_grad():
        for _ in range(2):
            logits, _, stats = m(idx)
        torch.cuda.synchronize()
        reps = 5
        e0, e1 = ev(), ev()
        e0.record()
        for _ in range(reps):
            logits, _, stats = m(idx)
        e1.record()
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    print(json.dumps(dict(config3=True, config='3: GPT 12x768 bf16, B=%d x T=%d, leaf 64, top-16, window 128' % (B, T),
                          forward_ms=ms, tokens_per_s=B * T / (ms * 1e-3), keys_per_query=stats['keys_total'],
                          data='synthetic (uniform random tokens, N(0,0.02) random-init weights)')), flush=True)


def run_prefill_attn(a, dev, emit=True):
    """Configuration 3, one layer of prefill sparse attention: B=4, H=12, T=8192, dh=64 bf16, 64-token leaves,
    top-16, 128-token window. q / k / v random, the selection from build_levels + select (the model's own
    kernels). Each launch is timed alone with CUDA events after a 256 MB L2 flush."""
    from treeattn_b200 import _ops
    from treeattn_b200._ops import Levels
    B = a.batch if a.batch != 64 else 4
    Hh, T, dh, leaf, topk, window = 12, 8192, 64, 64, 16, 128
    L0, Lm = 6, _ops.lm_of(T)
    g = torch.Generator(device=dev).manual_seed(11)
    q = torch.randn(B, Hh, T, dh, device=dev, generator=g).to(torch.bfloat16)
    k = (torch.randn(B, Hh, T, dh, device=dev, generator=g) * 0.5).to(torch.bfloat16)
    v = torch.randn(B, Hh, T, dh, device=dev, generator=g).to(torch.bfloat16)
    tq = torch.arange(T, device=dev)
    lv = Levels.empty(B, Hh, dh, T, L0, Lm, dev)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    ev = lambda: torch.cuda.Event(enable_timing=True)

    def timed(fn, reps):
        ts = []
        for r in range(reps + 1):
            flush.fill_(r & 0xff)
            e0, e1 = ev(), ev()
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            if r:
                ts.append(e0.elapsed_time(e1) * 1e3)
        return statistics.median(ts)

    sel_us = timed(lambda: (_ops.build_levels(k, T, L0, Lm, zero_sink=True, out=lv),
                            _ops.select(q, lv, tq, topk)), 3)
    ids, vld, _ = _ops.select(q, lv, tq, topk)
    ntree = 16
    out = torch.empty_like(q)
    if a.profile_steps:
        torch.cuda.cudart().cudaProfilerStart()
        for _ in range(a.profile_steps):
            _ops.build_levels(k, T, L0, Lm, zero_sink=True, out=lv)
            _ops.select(q, lv, tq, topk)
            _ops.prefill_attn(q, k, v, tq, ids, vld, ntree, leaf, window, dh ** -0.5, out=out, want_nkeys=False)
        torch.cuda.synchronize()
        torch.cuda.cudart().cudaProfilerStop()
        return
    _, _, nk = _ops.prefill_attn(q, k, v, tq, ids, vld, ntree, leaf, window, dh ** -0.5, out=out)
    tile_us = timed(lambda: _ops.prefill_attn(q, k, v, tq, ids, vld, ntree, leaf, window, dh ** -0.5, out=out,
                                              want_nkeys=False), 10)
    warp_us = timed(lambda: _ops.seg_attn(q, k, v, tq, ids, vld, ntree, leaf, window, dh ** -0.5, out=out,
                                          want_nkeys=False), 3)
    keys = float(nk.sum())
    flops = 4.0 * dh * keys
    pairs = union_tile_pairs(ids, vld, ntree, leaf, window, T)
    uflops = 4.0 * dh * 128 * 64 * pairs
    peaks = measured_peaks()
    peak = peaks['bf16_tflops'] if peaks else 1590.0
    line = dict(prefill_attn=True, config='3: B=%d H=12 T=8192 dh=64 bf16 leaf 64 top-16 window 128' % B,
                tile_kernel_us=tile_us, warp_kernel_us=warp_us, selection_us=sel_us,
                keys_per_query=keys / (B * Hh * T), algorithmic_flops=flops,
                achieved_tflops=flops / tile_us / 1e6, frac=flops / tile_us / 1e6 / peak,
                union_tile_pairs=pairs, union_flops=uflops, union_tflops=uflops / tile_us / 1e6,
                union_frac=uflops / tile_us / 1e6 / peak, warp_achieved_tflops=flops / warp_us / 1e6,
                peak_tflops=peak)
    if not a.no_cpu_baseline:
        line['cpu_baseline'] = cpu_prefill_sample(q, k, v, leaf, topk, window)
    if emit:
        print(json.dumps(line), flush=True)
    return line


def run_config1(a, dev, emit=True):
    """Configuration 1: GPT 4 layers, d=256, 4 heads, vocab 4096, T=512, leaf 32, top-4, window 64, fp32, batch 2,
    weights from torch.manual_seed(0) + GPT._init, tokens uniform from a seeded generator. The whole forward (our
    SegAttention path on the GPU) against the CPU oracle's forward (numpy fp32 restatement of model.py +
    fastseg.SegAttention) on the same weights and tokens: times and the max-abs logit difference (bound 1e-4 plus
    the reference's own fp32 noise at near-tied selections, which the parity tests pin separately)."""
    import numpy as np

    import oracle
    from treeattn_b200.config import Config
    from treeattn_b200.model import GPT
    cfg = Config(vocab_size=4096, seq_len=512, n_layer=4, n_head=4, n_embd=256, attn='seg', wmax=4, beam=4, local=64,
                 neighbors=False, beam_mode='fixed', leaf=32)
    torch.manual_seed(0)
    m = GPT(cfg).eval()
    idx = torch.randint(0, 4096, (2, 512), generator=torch.Generator().manual_seed(1))
    W = oracle.weights_from_state_dict({k: v.float() for k, v in m.state_dict().items()}, cfg.n_layer)
    m = m.to(dev)
    idx_d = idx.to(dev)
    ev = lambda: torch.cuda.Event(enable_timing=True)
    with torch.no_grad():
        for _ in range(3):
            logits, _, stats = m(idx_d)
        torch.cuda.synchronize()
        e0, e1 = ev(), ev()
        reps = 10
        e0.record()
        for _ in range(reps):
            logits, _, stats = m(idx_d)
        e1.record()
        torch.cuda.synchronize()
    gpu_ms = e0.elapsed_time(e1) / reps
    t0 = time.perf_counter()
    ref, rstats = oracle.gpt_forward(W, idx.numpy(), cfg.n_head, cfg.wmax, cfg.beam, cfg.local, L0=5)
    cpu_ms = (time.perf_counter() - t0) * 1e3
    diff = float(np.abs(logits.float().cpu().numpy() - ref).max())
    toks = 2 * 512
    line = dict(config1=True, config='1: GPT 4x256 fp32, B=2, T=512, leaf 32, top-4, window 64',
                gpu_forward_ms=gpu_ms, gpu_tokens_per_s=toks / (gpu_ms * 1e-3), max_abs_logit_diff=diff,
                keys_total=stats['keys_total'], ref_keys_total=rstats['keys_total'],
                cpu_baseline=dict(value=toks / (cpu_ms * 1e-3), unit='tokens/s', cores=_cpu_threads(), kind='port',
                                  sample='one full forward (2 x 512 tokens) of the CPU oracle in %.0f ms' % cpu_ms))
    if emit:
        print(json.dumps(line), flush=True)
    return line


def measure_kernels(a, dev, local):
    """The other configurations' hot kernels, measured after the configuration-4 decode loop so that one default
    run records them all (each with CUDA events and its own clock record): configuration 2's gather-dot,
    configuration 3's prefill attention layer (tensor-core tiles), configuration 5's decode kernel at the batch per
    GPU its engine runs (20 sequences of 32768 tokens) and configuration 1's whole forward."""
    import types
    base = dict(vars(a), profile_steps=0, cpu_seconds=min(a.cpu_seconds, 2.0), splits=0)
    out = {}

    def clocked(name, fn, **kw):
        ck = Clocks(local)
        ck.start()
        ck.mark_begin()
        line = fn(types.SimpleNamespace(**dict(base, **kw)), dev, emit=False)
        ck.mark_end()
        line['clocks'] = ck.stop()
        out[name] = line
        torch.cuda.empty_cache()

    clocked('config2_gather_dot', run_gather_dot)
    clocked('config3_prefill_layer', run_prefill_attn, batch=4)
    clocked('config5_decode_kernel', run_kernel_only, config5=True, batch=20, prompt=32768)
    clocked('config1_forward', run_config1)
    return out


def run_reference(a, rank, world):
    if rank != 0:
        return
    warm = max(0, a.warmup)
    value, steps, threads, how = cpu_decode_sample(max(5.0, a.cpu_seconds), seed=1)
    M = CFG4
    line = dict(metric=METRIC, value=value, unit='tokens/s', n_gpus=world, steps=a.steps, warmup=warm,
                ms_per_step=1000.0 / value, higher_is_better=True, scaling='weak', vs_baseline=None, dtype='f32',
                data='synthetic', impl='reference',
                config=dict(workload='config %s: KV-cache decode, %dx%d GPT bf16 (%d heads, vocab %d), batch '
                                     '%d/GPU, context %d, leaf %d, top-%d, window %d' % (
                                         M.name, M.NL, M.C, M.H, M.V, M.batch, M.prompt, M.leaf, M.topk, M.window),
                            global_batch=M.batch * world, seq_len=M.prompt,
                            parallelism='the CPU oracle (numpy restatement of the reference engine) on rank 0'),
                cpu_baseline=dict(value=value, unit='tokens/s', cores=threads, kind='port',
                                  sample='%s (12 layers + lm_head), fp32 numpy, cache filled with random K/V' % how),
                e2e=dict(value=value, unit='tokens/s', h2d_bytes_per_step=0, d2h_bytes_per_step=0))
    print(json.dumps(line), flush=True)


def main():
    a = parse()
    world = int(os.environ.get('WORLD_SIZE', '1'))
    rank = int(os.environ.get('RANK', '0'))
    local = int(os.environ.get('LOCAL_RANK', '0'))
    if a.impl == 'reference':
        run_reference(a, rank, world)
        return
    import torch.distributed as dist
    from treeattn_b200 import dist as tdist
    torch.cuda.set_device(local)
    dev = torch.device('cuda', local)
    if world > 1:
        tdist.init('nccl', timeout_s=600, device=dev)
    from treeattn_b200 import _ops
    from treeattn_b200.engine import Decoder
    if a.kernel_only:
        run_kernel_only(a, dev)
        return
    if a.gather_dot:
        run_gather_dot(a, dev)
        return
    if a.prefill_attn:
        run_prefill_attn(a, dev)
        return
    if a.config1:
        run_config1(a, dev)
        return
    if a.config3:
        run_config3(a, dev)
        return
    if a.dyn:
        run_dyn(a, dev)
        return
    if a.block:
        run_block(a, dev)
        return

    run_engine(a, CFG5 if a.config5 else CFG4, dev, rank, world, local)


def fill_random(dec, M, T0, seed):
    """Caches of every layer: positions [0, T0) from N(0, 0.25) keys and N(0, 1) values (bf16), trees built from
    them; every sequence at position T0 with a random token (configuration 5: a 32768-token prefill of 24 layers is
    not the measured step and the decode cost does not depend on the values)."""
    from treeattn_b200 import _ops
    g = torch.Generator(device=dec.dev).manual_seed(seed)
    for st in dec.states:
        for b in range(dec.batch):  # one sequence at a time: no full-size temporaries
            st.K[b, :, :T0].normal_(generator=g).mul_(0.5)
            st.V[b, :, :T0].normal_(generator=g)
        _ops.build_levels(st.K[:, :, :T0], st.cap, st.L0, st.Lm, zero_sink=True, out=st.levels)
    dec._tok.copy_(torch.randint(0, M.V, (dec.batch,), device=dec.dev, generator=g))
    dec._pos.fill_(T0)


def run_engine(a, M, dev, rank, world, local):
    """Greedy batched decoding of configuration 4 (default) or 5: timed device-resident loop, end-to-end serving
    loop, decode-kernel roofline, CPU-oracle baseline; one JSON line from rank 0."""
    import torch.distributed as dist
    from treeattn_b200 import _ops
    from treeattn_b200 import dist as tdist
    from treeattn_b200.engine import Decoder
    C, H, NL, dh = M.C, M.H, M.NL, M.dh
    B = a.batch if (a.batch != 64 or M is CFG4) else M.batch
    T0 = a.prompt if (a.prompt != 4096 or M is CFG4) else M.prompt
    K, Wm = a.steps if (a.steps != 256 or M is CFG4) else 128, max(a.warmup, 3)
    cap = ((T0 + Wm + 2 * K + 8 + M.leaf - 1) // M.leaf) * M.leaf
    cfg = make_cfg(M)
    W = make_weights(dev, 1234, torch.bfloat16, M)
    dec = Decoder(W, NL, H, C, M.tcap, 'seg', cfg, dev, batch=B, dtype=torch.bfloat16, cap=cap, splits=a.splits,
                  fused_linear=None if a.fused_linear < 0 else bool(a.fused_linear))
    torch.cuda.synchronize()
    t_pf = time.time()
    if M.fill == 'prefill':
        g = torch.Generator(device=dev).manual_seed(100 + rank)
        prompts = torch.randint(0, M.V, (B, T0), device=dev, generator=g)
        dec.prefill(prompts)
    else:
        fill_random(dec, M, T0, 100 + rank)
    torch.cuda.synchronize()
    t_pf = time.time() - t_pf
    if a.profile_steps:
        with torch.no_grad():
            for _ in range(Wm):
                dec._greedy_step()
            torch.cuda.synchronize()
            torch.cuda.cudart().cudaProfilerStart()
            for _ in range(a.profile_steps):
                dec._greedy_step()
            torch.cuda.synchronize()
            torch.cuda.cudart().cudaProfilerStop()
        print(json.dumps(dict(profile_steps=a.profile_steps, batch=B, splits=dec.splits,
                              keys_per_head=float(dec._nkeys.float().mean()))), flush=True)
        return
    dec._ensure_graphs()

    # ---------------------------------------------------------------- device-resident timed loop
    dec.greedy_steps(Wm)
    clocks = Clocks(local)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks.mark_begin()
    e0.record()
    dec.greedy_steps(K)
    e1.record()
    torch.cuda.synchronize()
    clocks.mark_end()
    ms = e0.elapsed_time(e1)
    ck = clocks.stop()
    if world > 1:
        dist.barrier()
    keys_mean = float(dec._nkeys.float().mean())

    # ---------------------------------------------------------------- end to end through the public API
    tok_host = torch.empty(B, dtype=torch.int64, pin_memory=True)
    tok_host.copy_(dec.tokens.cpu())
    dec.serve_step(tok_host, out=tok_host)  # warm-up
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record()
    for _ in range(K):
        dec.serve_step(tok_host, out=tok_host)
    f1.record()
    torch.cuda.synchronize()
    ms_e2e = f0.elapsed_time(f1)

    # ---------------------------------------------------------------- roofline: the fused decode kernel alone
    # The per-layer launches (one per layer cache, so consecutive launches read different KV and nothing stays
    # in L2) are captured in a CUDA graph and replayed, so the events see kernel time, not Python launch time.
    # Relaunching at the same position is idempotent (same appended row, same tree node).
    pos = dec.positions.clone()
    nk = torch.empty(B, H, device=dev, dtype=torch.int32)
    att = torch.empty(B, C, device=dev, dtype=torch.bfloat16)
    qkv = dec._qkv

    def layer_launches():
        for st in dec.states:
            _ops.decode_step(qkv, st.K, st.V, st.levels, pos, H, M.topk, M.topk, M.window, 1 / math.sqrt(dh), att,
                             nkeys=nk, splits=dec.splits, scratch=dec._split)

    layer_launches()
    torch.cuda.synchronize()
    kg, _ = dec._capture(layer_launches)
    kg.replay()
    torch.cuda.synchronize()
    reps = 10
    r0, r1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    r0.record()
    for _ in range(reps):
        kg.replay()
    r1.record()
    torch.cuda.synchronize()
    kern_ms = r0.elapsed_time(r1) / (reps * NL)
    sel_bytes = float(nk.sum()) * dh * 2 * 2  # K and V rows of the selected keys, bf16
    del kg

    # ---------------------------------------------------------------- reduce over ranks
    ms, ms_e2e, kern_ms = tdist.max_over_ranks([ms, ms_e2e, kern_ms], dev)
    if world > 1:
        tdist.gather_rows(dec.tokens.view(-1, 1))  # generated tokens gathered off the hot path

    # ---------------------------------------------------------------- strong scaling: the global batch fixed
    # The weak line above gives every rank the 1-GPU workload (B sequences); here the same B sequences are split
    # over the ranks (B / world each, engine.py:22-33: every sequence is independent), so the step time is that
    # of the smaller per-rank batch. Speed-up is against this run's own 1-GPU figure: each rank of the weak run is
    # exactly the 1-GPU configuration.
    strong = None
    if M is CFG4 and not a.no_strong and B % world == 0:
        if world == 1:
            strong = dict(global_batch=B, batch_per_rank=B, ms_per_step=ms / K, value=B * K / (ms * 1e-3),
                          unit='tokens/s', speedup=1.0, efficiency=1.0, note='the same run as value')
        else:
            del dec
            torch.cuda.empty_cache()
            Bs = B // world
            dec = Decoder(W, NL, H, C, M.tcap, 'seg', cfg, dev, batch=Bs, dtype=torch.bfloat16, cap=cap,
                          splits=a.splits, fused_linear=None if a.fused_linear < 0 else bool(a.fused_linear))
            g = torch.Generator(device=dev).manual_seed(100)
            prompts = torch.randint(0, M.V, (B, T0), device=dev, generator=g)  # the global batch, same on all ranks
            lo, hi = tdist.shard(B, rank, world)
            dec.prefill(prompts[lo:hi])
            dec._ensure_graphs()
            dec.greedy_steps(Wm)
            dist.barrier()
            torch.cuda.synchronize()
            s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s0.record()
            dec.greedy_steps(K)
            s1.record()
            torch.cuda.synchronize()
            ms_s = tdist.max_over_ranks([s0.elapsed_time(s1)], dev)[0]
            v_s = B * K / (ms_s * 1e-3)
            v_1 = B * K / (ms * 1e-3)  # every rank of the weak run decoded the whole 1-GPU batch
            strong = dict(global_batch=B, batch_per_rank=Bs, ms_per_step=ms_s / K, value=v_s, unit='tokens/s',
                          speedup=v_s / v_1, efficiency=v_s / v_1 / world, splits=dec.splits,
                          note='1-GPU reference: this run\'s weak-scaling step time (each rank decodes the whole '
                               '1-GPU batch of %d)' % B)
    if rank == 0:
        peaks = measured_peaks()
        peak = peaks['hbm_gbs'] if peaks else 6650.0
        achieved = sel_bytes / (kern_ms * 1e-3) / 1e9
        tokens = B * K * world
        kname = ('decode_persistent_kernel<bf16,%d>' % dh) if dec.splits < 0 else (
            'decode_kernel<bf16,%d> (%d CTA per (b, h))' % (dh, dec.splits))
        traffic = profiled_traffic() if M is CFG4 else None
        line = dict(metric=METRIC if M is CFG4 else METRIC5, value=tokens / (ms * 1e-3), unit='tokens/s',
                    n_gpus=world, steps=K, warmup=Wm, ms_per_step=ms / K, higher_is_better=True, scaling='weak',
                    vs_baseline=None, dtype='bf16',
                    data='synthetic (uniform random tokens, N(0,0.02) random-init weights%s)' % (
                        '' if M.fill == 'prefill' else '; caches filled with random keys/values'),
                    config=dict(workload='config %s: KV-cache decode, %dx%d GPT bf16 (%d heads, vocab %d), batch '
                                         '%d/GPU, context %d, leaf %d, top-%d, window %d' % (
                                             M.name, NL, C, H, M.V, B, T0, M.leaf, M.topk, M.window),
                                global_batch=B * world, seq_len=T0, parallelism='dp%d (batch sharded, no collective)'
                                % world, l2='inputs larger than L2 (KV cache %.1f GB/GPU)' % (
                                    2 * NL * B * H * cap * dh * 2 / 1e9),
                                prefill_s=round(t_pf, 2), keys_per_head=round(keys_mean, 1),
                                splits=dec.splits),
                    e2e=dict(value=tokens / (ms_e2e * 1e-3), unit='tokens/s', h2d_bytes_per_step=B * 8,
                             d2h_bytes_per_step=B * 8),
                    gpu_launches=(1 + NL * 4 + 1) * K,
                    roofline=dict(bound='hbm', achieved=achieved, peak=peak, unit='GB/s', frac=achieved / peak,
                                  traffic=traffic, traffic_source=(
                                      'profiles/decode_kernel_config4.md (ncu, same kernel and shape, t=4096)'
                                      if traffic else None),
                                  kernel='ta_decode_step (%s)' % kname,
                                  kernel_us=kern_ms * 1e3, bytes_per_launch=sel_bytes,
                                  peak_source='MEASURED_PEAKS.json hbm_gbs (burst copy)' if peaks else 'fallback'),
                    clocks=ck)
        if strong is not None:
            line['strong'] = strong
        if world == 1 and not a.no_cpu_baseline:
            v, steps, threads, how = cpu_decode_sample(a.cpu_seconds, W_dev=W if M is CFG4 else None, M=M)
            line['cpu_baseline'] = dict(value=v, unit='tokens/s', cores=threads, kind='port',
                                        sample=how + ' on the CPU oracle (numpy fp32 restatement of the reference '
                                        'engine), %s weights, cache filled with random K/V' % (
                                            'same' if M is CFG4 else 'random'))
        if world == 1 and M is CFG4 and not a.no_kernels:
            del dec
            torch.cuda.empty_cache()
            line['kernels'] = measure_kernels(a, dev, local)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == '__main__':
    main()
