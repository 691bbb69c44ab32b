"""Device faults surface through the layer API, not only through read_fault().

A fault is made without faulting the GPU: the expert-parallel rank barrier is
run for two ranks on one GPU with only rank 0 arriving (a flag nothing sets),
so its bounded wait gives up after its limit, sets fault bit 1 and returns;
the context stays usable.  The layer call that follows ends by copying the
fault word to the host, and the call after it raises DeviceFault before
launching anything.  check_faults() reports the same fault synchronously."""

from types import SimpleNamespace

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _layer():
    from spark_gpt_b200 import SparseMoE
    cfg = SimpleNamespace(hidden_size=256, num_experts=8, num_experts_per_tok=2,
                          moe_intermediate_size=128, norm_topk_prob=True)
    torch.manual_seed(0)
    m = SparseMoE(cfg).to(DEV)
    with torch.no_grad():
        m.gate.weight.normal_(0, 0.05)
        m.experts.gate_up_proj.normal_(0, 0.02)
        m.experts.down_proj.normal_(0, 0.02)
    return m


def _barrier_that_gives_up():
    from spark_gpt_b200 import ops
    flags = [torch.zeros(32, device=DEV, dtype=torch.int64) for _ in range(2)]
    table = torch.tensor([f.data_ptr() for f in flags], dtype=torch.int64, device=DEV)
    ops.ep_barrier(table, flags[0], 0, 2, 1)  # rank 1 never arrives
    return flags, table


def test_a_device_fault_raises_at_the_next_layer_call():
    from spark_gpt_b200 import DeviceFault, check_faults
    check_faults()  # start clean
    m = _layer()
    x = torch.randn(512, 256, device=DEV).to(torch.bfloat16)
    m(x)[0].float().sum().backward()
    torch.cuda.synchronize()

    keep = _barrier_that_gives_up()
    out = m(x)[0]          # runs; its closing snapshot copies the fault word
    torch.cuda.synchronize()
    with pytest.raises(DeviceFault, match="bounded device wait gave up"):
        m(x)
    del keep
    # raised once and cleared: training can resume after handling it
    out2 = m(x)[0]
    out2.float().sum().backward()
    torch.cuda.synchronize()
    check_faults()
    assert torch.isfinite(out.float()).all()


def test_check_faults_reports_synchronously():
    from spark_gpt_b200 import DeviceFault, check_faults
    check_faults()
    keep = _barrier_that_gives_up()
    with pytest.raises(DeviceFault) as ei:
        check_faults()
    assert ei.value.word == 1
    del keep
    check_faults()  # cleared
