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

V, C, H, NL = 50304, 768, 12, 12
LEAF, TOPK, WINDOW, TCAP = 64, 16, 128, 8192
# own kernels per greedy step: embed+LN; per layer the fused decode attention, 2 x add+LN and GELU; argmax+advance
# (the projections are cuBLAS)
OWN_LAUNCHES_PER_STEP = 1 + NL * 4 + 1
METRIC = 'decode tok/s (config 4: 12x768 bf16 GPT, batch 64/GPU, 4096-token prompts, leaf 64, top-16, window 128)'


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
                   help='with --kernel-only: the configuration-5 shape (dh 128, 128-token leaves, top-32, window 256, '
                        '32768-token context, Tcap 65536, 16 heads); --batch is per GPU (32 = 256 over 8 GPUs)')
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
    p.add_argument('--profile-steps', type=int, default=0,
                   help='profiling mode: after prefill and warm-up run this many eager decode steps between '
                        'cudaProfilerStart/Stop (for ncu --profile-from-start off) and exit')
    return p.parse_args()


def make_cfg(prompt, steps):
    from treeattn_b200.config import Config
    return Config(vocab_size=V, seq_len=TCAP, n_layer=NL, n_head=H, n_embd=C, attn='seg', wmax=TOPK, beam=TOPK,
                  local=WINDOW, neighbors=False, beam_mode='fixed', leaf=LEAF)


def make_weights(device, seed, dtype):
    """Random-init weights of the configuration-4 architecture (GPT._init: N(0, 0.02), c_proj 0.02/sqrt(2L))."""
    g = torch.Generator(device=device).manual_seed(seed)
    n = lambda *s, std=0.02: (torch.randn(*s, generator=g, device=device) * std).to(dtype)
    sp = 0.02 / math.sqrt(2 * NL)
    W = dict(wte=n(V, C), wpe=n(TCAP, C), ln_f=torch.ones(C, device=device), layers=[])
    for _ in range(NL):
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


def cpu_decode_sample(seconds, W_dev=None, seed=0):
    """Time the CPU oracle's decode (numpy, fp32, the reference engine's algorithm: engine.py:149-177 Decoder,
    batch 1) on the configuration-4 model for a bounded number of steps. The prompt cache (4096 positions per
    layer) is filled with random keys/values instead of a CPU prefill (the time of a decode step does not depend
    on the values). Returns (tokens/s, steps, threads)."""
    import numpy as np

    import oracle
    rng = np.random.default_rng(seed)
    if W_dev is not None:
        f = lambda t: t.float().cpu().numpy()
        W = dict(wte=f(W_dev['wte']), wpe=f(W_dev['wpe']), ln_f=f(W_dev['ln_f']),
                 layers=[{k: f(v) for k, v in L.items()} for L in W_dev['layers']])
    else:
        n = lambda *s, std=0.02: (rng.standard_normal(s, dtype=np.float32) * std)
        W = dict(wte=n(V, C), wpe=n(TCAP, C), ln_f=np.ones(C, np.float32),
                 layers=[dict(ln1=np.ones(C, np.float32), c_attn=n(3 * C, C), c_proj=n(C, C), ln2=np.ones(C, np.float32),
                              c_fc=n(4 * C, C), c_mlp=n(C, 4 * C)) for _ in range(NL)])
    T0 = 4096
    dec = oracle.DecoderNP(W, H, TCAP, TOPK, TOPK, WINDOW, L0=int(math.log2(LEAF)), cap=T0 + 512)
    dec.reset(1)
    for st in dec.states[0]:
        st.fill(rng.standard_normal((H, T0, C // H), dtype=np.float32),
                rng.standard_normal((H, T0, C // H), dtype=np.float32))
    tok = rng.integers(0, V, 1)
    dec.step(tok, T0)  # warm-up
    t0 = time.perf_counter()
    steps = 0
    while True:
        logits, _ = dec.step(tok, T0 + 1 + steps)
        tok = logits.argmax(-1)
        steps += 1
        if time.perf_counter() - t0 > seconds or steps >= 512:
            break
    dt = time.perf_counter() - t0
    return steps / dt, steps, _cpu_threads()


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


def run_kernel_only(a, dev):
    """Config-4 decode-attention kernel alone: batch a.batch x 12 heads, dh 64, bf16 caches holding a.prompt
    positions, leaf 64, top-16, window 128, position t = prompt (+ the launch index). With --profile-steps the
    launches are bracketed by cudaProfilerStart/Stop for ncu."""
    from treeattn_b200 import _ops
    from treeattn_b200._ops import Levels
    if a.config5:
        Hh, dh, leaf, topk, window, tcap = 16, 128, 128, 32, 256, 65536
        B, T0 = a.batch if a.batch != 64 else 32, 32768
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

    def run_all():
        for K, Vv, lv in layers:
            _ops.decode_step(qkv, K, Vv, lv, pos, Hh, topk, topk, window, 1 / math.sqrt(dh), att, nkeys=nk,
                             splits=splits)

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
    print(json.dumps(dict(kernel_only=True, config='5' if a.config5 else '4', batch=B, heads=Hh, dh=dh, prompt=T0,
                          splits=splits, kernel_us=us, bytes_per_launch=byts,
                          achieved_gbs=byts / us / 1e3, frac=byts / us / 1e3 / peak,
                          keys_per_head=float(nk.float().mean()))), flush=True)


def run_gather_dot(a, dev):
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
        _ops.gather_dot_blocks(q, K, blocks, blk, 0.125, nb_cta=2, out=out)
    torch.cuda.synchronize()
    if a.profile_steps:
        torch.cuda.cudart().cudaProfilerStart()
        for K in Ks[:a.profile_steps]:
            _ops.gather_dot_blocks(q, K, blocks, blk, 0.125, nb_cta=2, out=out)
        torch.cuda.synchronize()
        torch.cuda.cudart().cudaProfilerStop()
        return
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s), torch.cuda.graph(gr, stream=s):
        for K in Ks:
            _ops.gather_dot_blocks(q, K, blocks, blk, 0.125, nb_cta=2, out=out)
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
    print(json.dumps(line), flush=True)


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


def run_prefill_attn(a, dev):
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
    print(json.dumps(line), flush=True)


def run_reference(a, rank, world):
    if rank != 0:
        return
    warm = max(0, a.warmup)
    value, steps, threads = cpu_decode_sample(max(5.0, a.cpu_seconds), seed=1)
    line = dict(metric=METRIC, value=value, unit='tokens/s', n_gpus=world, steps=a.steps, warmup=warm,
                ms_per_step=1000.0 / value, higher_is_better=True, scaling='weak', vs_baseline=None, dtype='f32',
                data='synthetic', impl='reference',
                config=dict(workload='config 4 decode, CPU oracle (numpy restatement of the reference engine), '
                                     'batch 1 sample', global_batch=1, seq_len=4096, parallelism='none'),
                cpu_baseline=dict(value=value, unit='tokens/s', cores=threads, kind='port',
                                  sample='%d greedy decode steps of 1 sequence at t~4096 (12 layers + lm_head), '
                                         'fp32 numpy, cache filled with random K/V' % steps),
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

    B, T0, K, Wm = a.batch, a.prompt, a.steps, max(a.warmup, 3)
    cap = ((T0 + Wm + 2 * K + 8 + LEAF - 1) // LEAF) * LEAF
    cfg = make_cfg(T0, K)
    W = make_weights(dev, 1234, torch.bfloat16)
    dec = Decoder(W, NL, H, C, TCAP, 'seg', cfg, dev, batch=B, dtype=torch.bfloat16, cap=cap, splits=a.splits)
    g = torch.Generator(device=dev).manual_seed(100 + rank)
    prompts = torch.randint(0, V, (B, T0), device=dev, generator=g)
    torch.cuda.synchronize()
    t_pf = time.time()
    dec.prefill(prompts)
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
    # The 12 per-layer launches (one per layer cache, so consecutive launches read different KV and nothing stays
    # in L2) are captured in a CUDA graph and replayed, so the events see kernel time, not Python launch time.
    # Relaunching at the same position is idempotent (same appended row, same tree node).
    pos = dec.positions.clone()
    nk = torch.empty(B, H, device=dev, dtype=torch.int32)
    att = torch.empty(B, C, device=dev, dtype=torch.bfloat16)
    qkv = dec._qkv

    def layer_launches():
        for st in dec.states:
            _ops.decode_step(qkv, st.K, st.V, st.levels, pos, H, TOPK, TOPK, WINDOW, 1 / 8.0, att, nkeys=nk,
                             splits=dec.splits)

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
    sel_bytes = float(nk.sum()) * (C // H) * 2 * 2  # K and V rows of the selected keys, bf16
    del kg

    # ---------------------------------------------------------------- reduce over ranks
    ms, ms_e2e, kern_ms = tdist.max_over_ranks([ms, ms_e2e, kern_ms], dev)
    if world > 1:
        tdist.gather_rows(dec.tokens.view(-1, 1))  # generated tokens gathered off the hot path
    if rank == 0:
        peaks = measured_peaks()
        peak = peaks['hbm_gbs'] if peaks else 6650.0
        achieved = sel_bytes / (kern_ms * 1e-3) / 1e9
        tokens = B * K * world
        line = dict(metric=METRIC, value=tokens / (ms * 1e-3), unit='tokens/s', n_gpus=world, steps=K, warmup=Wm,
                    ms_per_step=ms / K, higher_is_better=True, scaling='weak', vs_baseline=None, dtype='bf16',
                    data='synthetic (uniform random tokens, N(0,0.02) random-init weights)',
                    config=dict(workload='config 4: KV-cache decode, 12x768 GPT bf16, batch %d/GPU, prompt %d, '
                                         'leaf %d, top-%d, window %d' % (B, T0, LEAF, TOPK, WINDOW),
                                global_batch=B * world, seq_len=T0, parallelism='dp%d (batch sharded, no collective)'
                                % world, l2='inputs larger than L2 (KV cache %.1f GB/GPU)' % (
                                    2 * NL * B * H * cap * (C // H) * 2 / 1e9),
                                prefill_s=round(t_pf, 2), keys_per_head=round(keys_mean, 1),
                                splits=dec.splits),
                    e2e=dict(value=tokens / (ms_e2e * 1e-3), unit='tokens/s', h2d_bytes_per_step=B * 8,
                             d2h_bytes_per_step=B * 8),
                    gpu_launches=OWN_LAUNCHES_PER_STEP * K,
                    roofline=dict(bound='hbm', achieved=achieved, peak=peak, unit='GB/s', frac=achieved / peak,
                                  traffic=profiled_traffic(), traffic_source='profiles/decode_kernel_config4.md (ncu, '
                                  'same kernel and shape, t=4096)',
                                  kernel='ta_decode_step (decode_persistent_kernel<bf16,64>)',
                                  kernel_us=kern_ms * 1e3, bytes_per_launch=sel_bytes,
                                  peak_source='MEASURED_PEAKS.json hbm_gbs (burst copy)' if peaks else 'fallback'),
                    clocks=ck)
        if world == 1 and not a.no_cpu_baseline:
            v, steps, threads = cpu_decode_sample(a.cpu_seconds, W_dev=W)
            line['cpu_baseline'] = dict(value=v, unit='tokens/s', cores=threads, kind='port',
                                        sample='%d greedy decode steps of 1 sequence at t~4096 on the CPU oracle '
                                               '(numpy fp32 restatement of the reference engine), same weights, '
                                               'cache filled with random K/V' % steps)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == '__main__':
    main()
