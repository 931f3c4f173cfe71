"""Paged KV cache: the paged write and paged split-K decode attention (t2c_kv_cache_write_paged,
t2c_attn_decode_paged) and the Qwen3 runner on a paged pool.

The paged write is byte movement: every row must land bit for bit where the
block table says.  Paged attention reads the same rows as the contiguous
kernel in the same order with the same split boundaries, so its output must be
bit-identical to t2c_attn_decode over the equivalent contiguous cache (and
within the fp32 tolerance of a plain softmax reference).  The runner on a
paged pool must give bit-identical layer outputs and greedy tokens to the
runner on contiguous caches with the same (unfused) kernels, and the oracle's
greedy tokens.
"""

from __future__ import annotations

import pytest
import torch

from test_decode_ops_gpu import _attn_ref, _close

pytestmark = pytest.mark.gpu


def _pool(B, NK, D, P, per_seq, seed):
    """A pool with sequence b's pages interleaved with the others' (page i of b at i * B + b, reversed)."""
    g = torch.Generator().manual_seed(seed)
    n_pages = B * per_seq + 3
    k = torch.randn(n_pages, P, NK, D, generator=g).half().cuda()
    v = torch.randn(n_pages, P, NK, D, generator=g).half().cuda()
    bt = torch.tensor([[n_pages - 1 - (i * B + b) for i in range(per_seq)] for b in range(B)], dtype=torch.int32)
    return k, v, bt.cuda()


def _gather(pages, bt):
    """Contiguous [B, S, NK, D] copy of each sequence's rows (host-side page walk)."""
    P = pages.shape[1]
    S = bt.shape[1] * P
    out = torch.zeros(bt.shape[0], S, *pages.shape[2:], dtype=pages.dtype, device=pages.device)
    for b in range(bt.shape[0]):
        for i, page in enumerate(bt[b].tolist()):
            out[b, i * P:(i + 1) * P] = pages[page]
    return out


@pytest.mark.parametrize("P", [16, 64])
@pytest.mark.parametrize("T", [1, 37])
def test_kv_cache_write_paged_is_exact(P, T):
    from torch2vk_b200 import kernels

    B, NK, D, per_seq = 3, 8, 128, 6
    k, _, bt = _pool(B, NK, D, P, per_seq, seed=1)
    before = k.clone()
    positions = torch.tensor([0, P - 1, 3 * P + 5], dtype=torch.int32, device="cuda")
    src = torch.randn(B, T, NK * D, device="cuda").half()
    kernels.device_status(clear=True)
    kernels.kv_cache_write_paged(k, src, positions, bt, batch=B, tokens=T, n_kv=NK, head_dim=D)
    torch.cuda.synchronize()
    assert kernels.device_status() == 0
    want = before.clone()
    for b in range(B):
        for t in range(T):
            pos = int(positions[b]) + t
            want[bt[b, pos // P], pos % P] = src[b, t].view(NK, D)
    assert torch.equal(k, want)


@pytest.mark.parametrize("NH,NK,D", [(32, 8, 128), (16, 8, 128), (16, 16, 64)])
@pytest.mark.parametrize("splits", [1, 5, 16])
def test_attn_decode_paged_matches_contiguous(NH, NK, D, splits):
    from torch2vk_b200 import kernels

    B, P, per_seq = 4, 32, 24
    k, v, bt = _pool(B, NK, D, P, per_seq, seed=2)
    S = per_seq * P
    positions = torch.tensor([0, 31, 400, S - 1], dtype=torch.int32, device="cuda")
    q = torch.randn(B, NH * D, device="cuda").half()
    kernels.device_status(clear=True)
    got = kernels.attn_decode_paged(q, k, v, positions, bt, batch=B, n_heads=NH, n_kv=NK, head_dim=D, splits=splits)
    kc, vc = _gather(k, bt), _gather(v, bt)
    want = kernels.attn_decode(q, kc, vc, positions, batch=B, n_heads=NH, n_kv=NK, head_dim=D, max_len=S,
                               splits=splits)
    torch.cuda.synchronize()
    assert kernels.device_status() == 0
    assert torch.equal(got, want)
    lens = [int(p) + 1 for p in positions]
    _close(got.view(B, NH, D), _attn_ref(q.view(B, NH, D), kc, vc, lens, NH, NK))


def test_paged_bad_table_entry_is_reported():
    """A block-table entry outside the pool: the write skips that row, attention reads page 0 in its place, and
    both report T2C_EINVAL in the device status; the other sequences are unaffected."""
    from torch2vk_b200 import kernels

    B, NH, NK, D, P, per_seq = 2, 16, 8, 128, 16, 4
    k, v, bt = _pool(B, NK, D, P, per_seq, seed=3)
    bt[1, 1] = k.shape[0] + 5
    positions = torch.tensor([40, 20], dtype=torch.int32, device="cuda")
    before = k.clone()
    kernels.device_status(clear=True)
    src = torch.randn(B, 1, NK * D, device="cuda").half()
    kernels.kv_cache_write_paged(k, src, positions, bt, batch=B, tokens=1, n_kv=NK, head_dim=D)
    torch.cuda.synchronize()
    assert kernels.device_status(clear=True) & (1 << 1)
    want = before.clone()
    want[bt[0, 40 // P], 40 % P] = src[0, 0].view(NK, D)
    assert torch.equal(k, want)
    q = torch.randn(B, NH * D, device="cuda").half()
    out = kernels.attn_decode_paged(q, k, v, positions, bt, batch=B, n_heads=NH, n_kv=NK, head_dim=D, splits=2)
    torch.cuda.synchronize()
    assert kernels.device_status(clear=True) & (1 << 1)
    kc, vc = _gather(k, bt[:1]), _gather(v, bt[:1])
    _close(out.view(B, NH, D)[:1], _attn_ref(q.view(B, NH, D)[:1], kc, vc, [41], NH, NK))


def test_paged_rejects_bad_arguments():
    from torch2vk_b200 import kernels

    B, NH, NK, D, P = 1, 16, 8, 128, 16
    k, v, bt = _pool(B, NK, D, P, 2, seed=4)
    q = torch.zeros(B, NH * D, device="cuda").half()
    pos = torch.zeros(B, dtype=torch.int32, device="cuda")
    k3 = torch.zeros(4, 24, NK, D, device="cuda").half()
    with pytest.raises(RuntimeError, match="power of two"):
        kernels.attn_decode_paged(q, k3, k3, pos, bt, batch=B, n_heads=NH, n_kv=NK, head_dim=D)
    with pytest.raises(RuntimeError, match="workspace"):
        kernels.attn_decode_paged(q, k, v, pos, bt, batch=B, n_heads=NH, n_kv=NK, head_dim=D, splits=4,
                                  workspace=torch.empty(8, device="cuda"))


def test_qwen3_runner_paged_matches_contiguous_and_oracle():
    """Batch 3, a 40-token prompt, 24 greedy steps with the decode graph: the paged runner (pages of 16,
    interleaved between sequences) against the contiguous runner with the same unfused attention kernels,
    bit for bit, and against the oracle's greedy ids."""
    from oracle import qwen3_ref
    from test_qwen3_gpu import SMALL, upload
    from torch2vk_b200.qwen3 import Qwen3Config, Qwen3Runner

    cfg = Qwen3Config(**SMALL)
    pm = qwen3_ref.build(cfg.hidden, cfg.layers, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.intermediate, cfg.vocab,
                         seed=0, topology="q4_k_m")
    ids = qwen3_ref.prompt_ids(40, cfg.vocab, seed=0, batch=3)
    w = upload(pm, cfg)
    common = dict(batch=3, max_seq=128, max_new_tokens=25, decode_splits=4, fused_attention=False)
    paged = Qwen3Runner(cfg, w, page_size=16, **common)
    flat = Qwen3Runner(cfg, w, **common)
    outs_p: list[torch.Tensor] = []
    outs_f: list[torch.Tensor] = []
    paged.prefill(ids.cuda(), layer_outputs=outs_p)
    flat.prefill(ids.cuda(), layer_outputs=outs_f)
    for a, b in zip(outs_p, outs_f):
        assert torch.equal(a, b)
    pages = paged.paged.pages(0)
    assert pages != list(range(pages[0], pages[0] + len(pages)))  # not one contiguous run
    outs_p, outs_f = [], []
    paged.decode_step(layer_outputs=outs_p)
    flat.decode_step(layer_outputs=outs_f)
    for a, b in zip(outs_p, outs_f):
        assert torch.equal(a, b)
    got = paged.generate(ids.cuda(), 24).cpu()
    assert torch.equal(got, flat.generate(ids.cuda(), 24).cpu())
    # against the oracle: identical up to the first step whose top-two logit gap (over the batch) is below
    # 0.02, where fp16-activation rounding may legitimately pick the other token (this seed: step 15)
    ref, gaps = qwen3_ref.greedy(pm.hf, ids, 24)
    n = next((i for i, gap in enumerate(gaps) if gap < 0.02), 24)
    assert n >= 12, gaps
    assert torch.equal(got[:, :n], ref[:, :n]), f"paged {got.tolist()}\nref {ref.tolist()}\nmin top-2 gaps {gaps}"
    from torch2vk_b200 import kernels

    assert kernels.device_status() == 0
