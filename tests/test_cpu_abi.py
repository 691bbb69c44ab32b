"""CPU-side checks: the C-ABI library loads here (no GPU) and exports every
entry point include/b200moe.h declares; host helpers; the Python mirror of
the reference interface (names, shapes, loud failure without CUDA)."""

import re
from pathlib import Path
from types import SimpleNamespace

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]


def header_functions():
    text = (ROOT / "include" / "b200moe.h").read_text()
    return sorted(set(re.findall(r"\b(b200moe_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from spark_gpt_b200 import _lib
    from spark_gpt_b200.build import build
    build()
    return _lib.load()


def test_library_exports_every_header_symbol(lib):
    from spark_gpt_b200 import _lib
    names = header_functions()
    assert len(names) >= 25
    for n in names:
        assert hasattr(lib, n), n
        assert n in _lib.PROTOTYPES, n
    assert set(_lib.PROTOTYPES) == set(names)


def test_host_helpers(lib):
    assert lib.b200moe_version() >= 100
    pr = lib.b200moe_padded_rows
    for R, E in [(0, 1), (1, 1), (524288, 64), (131072, 128), (21, 5)]:
        v = pr(R, E)
        assert v % 128 == 0 and v >= R + E * 127 and v < R + E * 127 + 128
    assert [lib.b200moe_router_width(e) for e in (1, 8, 64, 65, 128, 129, 256)] == \
        [64, 64, 64, 128, 128, 256, 256]
    from spark_gpt_b200 import _lib
    assert _lib.value("b200moe_dispatch_scratch_bytes", 65536, 8, 64) == 128 * 64 * 4
    # load-balance statistics: 1184 block partial rows (8 per SM of 148), then
    # 37 level-one sums of 32 rows, 2E+2 floats each
    assert _lib.value("b200moe_lb_scratch_bytes", 65536, 64) == (1184 + 37) * 130 * 4
    assert _lib.value("b200moe_lb_scratch_bytes", 100, 64) == (4 + 1) * 130 * 4  # 32 tokens a block


def test_entry_points_reject_bad_arguments_without_touching_the_gpu(lib):
    from spark_gpt_b200 import _lib
    with pytest.raises(RuntimeError, match="null pointer"):
        _lib.call("b200moe_router_topk_fwd", None, 0, 64, 10, 64, 8, 1, None, None, None)
    with pytest.raises(RuntimeError, match="k <="):
        _lib.call("b200moe_router_topk_fwd", 16, 0, 64, 10, 64, 17, 1, 16, 16, None)
    with pytest.raises(RuntimeError, match="multiple of 128"):
        _lib.call("b200moe_expert_down_fwd", 16, 16, 16, 16, None, 1024, 8, 200, 64, 16, None)
    with pytest.raises(RuntimeError, match="I must be"):
        _lib.call("b200moe_expert_gate_up_fwd", 16, 16, 16, 16, 1024, 8, 256, 100, 16, 16, None)
    with pytest.raises(RuntimeError, match="scratch too small"):
        _lib.call("b200moe_dispatch", 16, 1000, 8, 64, 16, 16, 16, 16, 16, 16, 16, 4, None)
    with pytest.raises(RuntimeError, match="segments"):
        _lib.call("b200moe_expert_wgrad_segments", 16, 512, 16, 256, 16, 0, 8, 1024, 16, 0, None)
    with pytest.raises(RuntimeError, match="N must be"):
        _lib.call("b200moe_expert_wgrad_segments", 16, 512, 16, 100, 16, 2, 8, 1024, 16, 0, None)


def _cfg():
    return SimpleNamespace(hidden_size=256, num_experts=8, num_experts_per_tok=2,
                           moe_intermediate_size=128, norm_topk_prob=True)


def test_module_mirrors_reference_parameter_layout():
    from spark_gpt_b200 import SparseMoE
    m = SparseMoE(_cfg())
    shapes = {n: tuple(p.shape) for n, p in m.named_parameters()}
    assert shapes == {"gate.weight": (8, 256), "experts.gate_up_proj": (8, 256, 256),
                      "experts.down_proj": (8, 256, 128)}
    assert all(p.dtype == torch.float32 for p in m.parameters())
    assert m.experts.num_experts == 8 and m.experts.hidden_dim == 256
    assert m.experts.intermediate_dim == 128
    assert tuple(m.experts.fp8_scale.shape) == (5,)
    # state_dict keys are what export_hf passes through (train.py:2548-2559)
    assert set(m.state_dict()) == {"gate.weight", "experts.gate_up_proj", "experts.down_proj"}


def test_no_cpu_fallback():
    from spark_gpt_b200 import SparseMoE
    m = SparseMoE(_cfg())
    with pytest.raises(RuntimeError, match="no CPU path"):
        m(torch.randn(4, 256))


def test_row_arena_layout(lib):
    """The pipelined expert-parallel layer's shared row buffers: chunk s owns
    rows [base_s, base_s + cap_s) in source order, capacities are the chunks'
    dispatch capacities (none for a chunk without rows or slots), and the
    segment table moves each chunk's padded expert offsets to its base."""
    from spark_gpt_b200 import ops
    from spark_gpt_b200.ep import RowArena
    E = 4
    arena = RowArena.for_chunks([10, 0, 7, 3], [25, 0, 9, 0], E, "cpu")
    caps = [ops.padded_rows(25, E), 0, ops.padded_rows(9, E), 0]
    assert arena.caps == caps and all(c % 128 == 0 for c in caps)
    assert arena.base == [0, caps[0], caps[0], caps[0] + caps[2]]
    assert arena.total == sum(caps)
    arena.alloc("xs", 16)
    assert arena.bufs["xs"].shape == (sum(caps), 16)
    assert arena.rows("xs", 1).shape == (0, 16)
    v = arena.rows("xs", 2)
    assert v.shape == (caps[2], 16) and v.is_contiguous()
    assert v.data_ptr() == arena.bufs["xs"].data_ptr() + caps[0] * 16 * 2
    i32 = torch.int32
    d0 = SimpleNamespace(pad_offsets=torch.tensor([0, 128, 128, 256, 384], dtype=i32))
    d2 = SimpleNamespace(pad_offsets=torch.tensor([0, 0, 128, 128, 128], dtype=i32))
    segs = arena.segments([d0, None, d2, None], E)
    assert segs.dtype == i32 and segs.shape == (4, E + 1)
    assert segs[0].tolist() == [0, 128, 128, 256, 384]
    assert segs[1].tolist() == [caps[0]] * (E + 1)
    assert segs[2].tolist() == [caps[0] + x for x in (0, 0, 128, 128, 128)]
    assert segs[3].tolist() == [caps[0] + caps[2]] * (E + 1)
    # per expert: the union of its segments holds every chunk's padded rows
    lens = (segs[:, 1:] - segs[:, :-1]).sum(0).tolist()
    assert lens == [128, 128, 128, 128]
    # an arena without rows still has one 128-row block to hand out
    assert RowArena.for_chunks([0, 0], [0, 0], E, "cpu").total == 128
