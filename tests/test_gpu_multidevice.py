"""Two GPUs driven from one process. The library keeps some launch state per device: the dynamic shared-memory
size allowed for each kernel, the decode kernel's CTAs per SM and the SM count. The same work on cuda:0 and then
on cuda:1 must therefore run on both and give identical results. The kernels run on the current CUDA device (as
the reference's launches do), so each half runs under torch.cuda.device. Skipped with fewer than two GPUs."""
import pytest
import torch

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                                 reason='needs two GPUs')]


def _decode(dev):
    """Prefill + 48 batched decode steps of a small bf16 GPT: the persistent decode kernel (113 KB of shared
    memory at this shape), the appends and the tree updates."""
    from treeattn_b200.config import Config
    from treeattn_b200.engine import Decoder, weights_from_ours
    from treeattn_b200.model import GPT
    cfg = Config(vocab_size=128, seq_len=512, n_layer=2, n_head=4, n_embd=256, attn='seg', wmax=8, beam=8,
                 beam_classes=(2, 4, 8), local=64, leaf=32, beam_mode='fixed', neighbors=False)
    torch.manual_seed(3)
    m = GPT(cfg).eval()
    W = weights_from_ours({k: v.to(torch.bfloat16) for k, v in m.state_dict().items()}, cfg)
    idx = torch.randint(0, 128, (48, 304), generator=torch.Generator().manual_seed(5))
    with torch.cuda.device(dev):
        dec = Decoder(W, cfg.n_layer, cfg.n_head, cfg.n_embd, 512, 'seg', cfg, dev, batch=48, dtype=torch.bfloat16)
        dec.prefill(idx[:, :256].to(dev))
        out = [dec.step(idx[:, t].to(dev), t)[0].float().cpu() for t in range(256, 304)]
    return torch.stack(out)


def _select(dev):
    """Dynamic-tree select_keys: the 2-means build (CTA and subtree kernels) and the select loop (64 KB of shared
    memory)."""
    from treeattn_b200.config import Config
    from treeattn_b200.dyntree import select_keys
    g = torch.Generator().manual_seed(9)
    q = torch.randn(1, 4, 1024, 64, generator=g)
    k = torch.randn(1, 4, 1024, 64, generator=g)
    lhat = torch.randint(2, 9, (1, 4, 1024), generator=g)
    cfg = Config(attn='dyn', seq_len=1024, chunk=64, wmax=8, neighbors=True)
    with torch.cuda.device(dev):
        sel = select_keys(q.to(dev), k.to(dev), lhat.to(dev), cfg)
        return {key: v.cpu() for key, v in sel.items()}


def test_decode_same_on_two_devices():
    a = _decode('cuda:0')
    b = _decode('cuda:1')
    assert torch.equal(a, b)


def test_select_keys_same_on_two_devices():
    a = _select('cuda:0')
    b = _select('cuda:1')
    for key in a:
        assert torch.equal(a[key], b[key]), key
    from treeattn_b200 import _ops
    for dev in (0, 1):
        with torch.cuda.device(dev):
            assert _ops.device_error()[0] == 0
