"""The persistent schedule: CTAs that process several work items in a row.

The grid has one CTA per SM and each CTA walks its items (256 query rows of one head)
one after another, so the cases here have several items per CTA:

* an odd number of K/V tiles per item, which moves the ring phase of every later item
  of the CTA (its first K sits in slot 2 instead of 0);
* causal items of different lengths (2, 4 and 5 tiles) mixed in one CTA;
* items that see no key at all (n_tiles = 0) between items that do;
* an output that is not 32-byte aligned, which takes the 16-byte store path.

Results are compared with the fp64 oracle on the same bf16 inputs (every head, or
every 25th head where a plain PyTorch fp32 reference on the GPU checks all of them) under
the usual tolerances (max-abs 2e-2, mean-abs 2e-3, LSE 1e-3).
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import attention_oracle as oracle

pytestmark = pytest.mark.gpu


def _check(out, lse, ref_o, ref_lse):
    metrics = oracle.error_metrics(out, ref_o, lse, ref_lse)
    assert np.isfinite(out).all()
    assert metrics["max_abs"] <= oracle.MAX_ABS_TOL, metrics
    assert metrics["mean_abs"] <= oracle.MEAN_ABS_TOL, metrics
    assert metrics["lse_max_abs"] <= oracle.LSE_TOL, metrics
    assert np.array_equal(np.isneginf(lse), np.isneginf(ref_lse))


@pytest.mark.parametrize(
    "shape,causal",
    [
        ((2, 150, 384, 128), False),   # 600 items of 3 tiles: the ring phase flips every item
        ((1, 200, 640, 128), True),    # 600 causal items of 5, 4 and 2 tiles
        ((1, 160, 333, 128), False),   # ragged: 3 tiles with a partial last one, partial rows
    ],
)
def test_several_items_per_cta(b200, shape, causal):
    import torch

    assert shape[0] * shape[1] * ((shape[2] + 255) // 256) > 2 * 148
    from avo.benchmark import error_metrics, fp32_reference

    q, k, v = oracle.make_inputs(shape, seed=21)
    dq, dk, dv = (t.cuda() for t in (q, k, v))
    out, lse = b200.attention_forward(dq, dk, dv, causal)
    torch.cuda.synchronize()
    b200.check_status(dq.device)
    # Every head against the plain PyTorch fp32 reference on the GPU ...
    ref_o, ref_lse = fp32_reference(dq, dk, dv, causal)
    metrics = error_metrics(out, ref_o, lse, ref_lse)
    assert metrics["max_abs"] <= oracle.MAX_ABS_TOL, metrics
    assert metrics["mean_abs"] <= oracle.MEAN_ABS_TOL, metrics
    assert metrics["lse_max_abs"] <= oracle.LSE_TOL, metrics
    # ... and every 25th head against the fp64 oracle.
    seq = shape[2]
    pick = slice(None, None, 25)
    heads = [t.reshape(-1, seq, 128)[pick].float().numpy() for t in (q, k, v)]
    ref_o, ref_lse = oracle.attention_fp64(*heads, causal)
    _check(out.reshape(-1, seq, 128)[pick].float().cpu().numpy(), lse.reshape(-1, seq)[pick].cpu().numpy(),
           ref_o, ref_lse)


def _rand_bf16(shape, seed):
    import torch

    g = torch.Generator().manual_seed(seed)
    return torch.randn(shape, generator=g).to(torch.bfloat16)


def test_items_without_keys_between_items(b200):
    import torch

    # Query rows 0-511 at positions 0-511, keys at positions 300-683: the first 256-row
    # block of every head sees no key (an item with no tiles), the second sees some.
    bh, seq_q, seq_kv, q_pos0, kv_pos0 = 150, 512, 384, 0, 300
    q = _rand_bf16((bh, seq_q, 128), 31).cuda()
    k = _rand_bf16((bh, seq_kv, 128), 32).cuda()
    v = _rand_bf16((bh, seq_kv, 128), 33).cuda()
    out = torch.full((bh, seq_q, 128), 7.0, dtype=torch.bfloat16, device="cuda")
    lse = torch.full((bh, seq_q), 7.0, dtype=torch.float32, device="cuda")
    b200.attention_block(q, k, v, out, lse, causal=True, q_pos0=q_pos0, kv_pos0=kv_pos0)
    torch.cuda.synchronize()
    b200.check_status("cuda:0")
    ref_o, ref_lse = oracle.attention_fp64(q.float().cpu().numpy(), k.float().cpu().numpy(),
                                           v.float().cpu().numpy(), True, q_pos0=q_pos0, kv_pos0=kv_pos0)
    got_lse = lse.cpu().numpy()
    assert np.isneginf(got_lse[:, :300]).all()
    assert torch.all(out[:, :300] == 0)
    _check(out.float().cpu().numpy(), got_lse, ref_o, ref_lse)


def test_output_not_32_byte_aligned(b200):
    import torch

    # O starts 8 elements (16 bytes) into its buffer and heads are seq*128 + 8 elements
    # apart, so neither the base nor the head stride is a multiple of 32 bytes.
    bh, seq = 160, 384
    q = _rand_bf16((bh, seq, 128), 41).cuda()
    k = _rand_bf16((bh, seq, 128), 42).cuda()
    v = _rand_bf16((bh, seq, 128), 43).cuda()
    stride = seq * 128 + 8
    buf = torch.full((8 + bh * stride + 8,), 7.0, dtype=torch.bfloat16, device="cuda")
    out = torch.as_strided(buf, (bh, seq, 128), (stride, 128, 1), storage_offset=8)
    lse = torch.empty((bh, seq), dtype=torch.float32, device="cuda")
    assert out.data_ptr() % 32 == 16
    b200.attention_block(q, k, v, out, lse, causal=False, q_pos0=0, kv_pos0=0)
    torch.cuda.synchronize()
    b200.check_status("cuda:0")
    ref_o, ref_lse = oracle.attention_fp64(q.float().cpu().numpy(), k.float().cpu().numpy(),
                                           v.float().cpu().numpy(), False)
    _check(out.float().cpu().numpy(), lse.cpu().numpy(), ref_o, ref_lse)
    # The gaps between heads and the ends of the buffer were not written.
    host = buf.float().cpu().numpy()
    assert (host[:8] == 7.0).all() and (host[-8:] == 7.0).all()
    gaps = np.stack([host[8 + h * stride + seq * 128: 8 + (h + 1) * stride] for h in range(bh - 1)])
    assert (gaps == 7.0).all()
