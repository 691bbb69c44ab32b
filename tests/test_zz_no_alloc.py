"""b200moe_dispatch_noalloc: dispatch for callers that cannot allocate device memory.

Some callers of this library hold only their input and output buffers: a host runtime
bound through FFI that owns a fixed device arena and has no caching allocator, or code
that must not call cudaMalloc/cudaFree because those can synchronize the device or fail
under memory pressure in the middle of a step.  This entry point gives them the dispatch
without the caller-provided scratch: its per-chunk counts live in a fixed 1 MiB array
built into the library.  The checks here call both entry points through the C ABI and
require identical outputs (dispatch is integer work: bit-exact), over two calls in a row
so that what the first call leaves in the shared array cannot leak into the second.
This file is named so that pytest collects it last.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _outputs(T, k, E):
    from spark_gpt_b200 import _lib
    cap = int(_lib.value("b200moe_padded_rows", T * k, E))
    i32 = dict(device=DEV, dtype=torch.int32)
    return {
        "counts": torch.full((E,), -7, **i32),
        "offsets": torch.full((E,), -7, **i32),
        "pad_offsets": torch.full((E + 1,), -7, **i32),
        "row_flat": torch.full((cap,), -7, **i32),
        "inv_pad": torch.full((max(T * k, 1),), -7, **i32),
        "tile_expert": torch.full((cap // 128,), -7, **i32),
    }


def _args(o):
    return [_p(o[n]) for n in ("counts", "offsets", "pad_offsets", "row_flat", "inv_pad",
                               "tile_expert")]


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def dispatch_with_scratch(sel, E):
    from spark_gpt_b200 import _lib
    T, k = sel.shape
    o = _outputs(T, k, E)
    nbytes = int(_lib.value("b200moe_dispatch_scratch_bytes", T, k, E))
    scratch = torch.empty(nbytes, device=DEV, dtype=torch.uint8)
    _lib.call("b200moe_dispatch", _p(sel), T, k, E, *_args(o), _p(scratch), nbytes, _stream())
    return o


def dispatch_noalloc(sel, E):
    from spark_gpt_b200 import _lib
    T, k = sel.shape
    o = _outputs(T, k, E)
    _lib.call("b200moe_dispatch_noalloc", _p(sel), T, k, E, *_args(o), _stream())
    return o


def _routing(T, k, E, seed, skew):
    g = torch.Generator().manual_seed(seed)
    p = torch.ones(E)
    if skew:
        p[: E // 4] = 0.0
        p[-1] = 30.0
    sel = torch.stack([torch.multinomial(p, k, replacement=False, generator=g) for _ in range(T)])
    return sel.to(DEV).contiguous()


def _same(a, b):
    n = int(a["pad_offsets"][-1])
    assert int(b["pad_offsets"][-1]) == n
    for key in ("counts", "offsets", "pad_offsets", "inv_pad"):
        assert torch.equal(a[key], b[key]), key
    assert torch.equal(a["row_flat"][:n], b["row_flat"][:n])
    assert torch.equal(a["tile_expert"][: n // 128], b["tile_expert"][: n // 128])


def test_noalloc_dispatch_matches_dispatch_on_two_calls_in_a_row():
    from spark_gpt_b200 import _lib
    # first call: many chunks, skewed routing; second: a different, smaller routing
    first = _routing(20000, 8, 64, seed=1, skew=True)
    second = _routing(3000, 4, 16, seed=2, skew=False)
    for sel, E in ((first, 64), (second, 16)):
        ref = dispatch_with_scratch(sel, E)
        got = dispatch_noalloc(sel, E)
        torch.cuda.synchronize()
        _same(ref, got)
    # and again on the first input, after the second call changed the shared array
    _same(dispatch_with_scratch(first, 64), dispatch_noalloc(first, 64))
    torch.cuda.synchronize()
    assert _lib.read_fault() == 0


def test_noalloc_dispatch_rejects_sizes_beyond_its_scratch():
    from spark_gpt_b200 import _lib
    T, k, E = 600_000, 8, 256  # ceil(4.8M / 4096) * 256 = 300,032 > 262,144 counts
    sel = torch.zeros(1, dtype=torch.int64, device=DEV)
    o = _outputs(1, 1, E)
    with pytest.raises(RuntimeError, match="built-in scratch holds 262144"):
        _lib.call("b200moe_dispatch_noalloc", _p(sel), T, k, E, *_args(o), _stream())
