"""The custom-op registration of the fused layer, checked without a GPU.

The fake (meta) implementations must give the shapes and dtypes the CUDA
implementation returns, so that torch.compile can trace SparseMoE (as
train.py:3787 compiles the model) without running it; the symbolic padded
capacity must equal the library's own b200moe_padded_rows.
"""

import torch
from torch._subclasses.fake_tensor import FakeTensorMode

from spark_gpt_b200 import _lib, ops
from spark_gpt_b200.custom_ops import padded_capacity


def test_padded_capacity_matches_library():
    _lib.load()
    for R in (0, 1, 127, 128, 129, 4096, 65536 * 8 + 3):
        for E in (1, 8, 64, 128, 256):
            assert padded_capacity(R, E) == ops.padded_rows(R, E)


def test_fake_forward_and_backward_shapes():
    T, H, E, K, I = 100, 256, 8, 2, 128
    with FakeTensorMode():
        dev = "cuda"
        x = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
        wr = torch.empty(E, H, device=dev)
        wgu = torch.empty(E, 2 * I, H, device=dev)
        wd = torch.empty(E, H, I, device=dev)
        outs = torch.ops.b200moe.sparse_moe_fwd(x, wr, wgu, wd, K, True)
        out, logits_buf, sel, wr_b, wgu_b, wd_b, rw, xs, gu, h, y = outs[:11]
        counts, offsets, pad_offsets, row_flat, inv_pad, tile_expert = outs[11:]
        cap = padded_capacity(T * K, E)
        W = 64
        assert out.shape == (T, H) and out.dtype == torch.bfloat16
        assert logits_buf.shape == (T, W) and sel.shape == (T, K) and sel.dtype == torch.int64
        assert (wr_b.shape, wgu_b.shape, wd_b.shape) == ((W, H), (E, 2 * I, H), (E, H, I))
        assert xs.shape == (cap, H) and gu.shape == (cap, 2 * I) and h.shape == (cap, I)
        assert y.shape == (cap, H) and rw.shape == (T, K)
        assert counts.shape == (E,) and pad_offsets.shape == (E + 1,)
        assert row_flat.shape == (cap,) and inv_pad.shape == (T * K,)
        assert tile_expert.shape == (cap // 128,)
        d_out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
        dx, g_r, g_gu, g_d = torch.ops.b200moe.sparse_moe_bwd(
            d_out, None, x, *outs[1:], K, True, E)
        assert dx.shape == (T, H) and g_r.shape == (E, H)
        assert g_gu.shape == (E, 2 * I, H) and g_d.shape == (E, H, I)
        assert g_gu.dtype == torch.float32
