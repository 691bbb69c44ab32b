"""bench.py's reference arm on the CPU: one JSON line with the contract's keys
(the driver parses it), on a tiny token sample so the test stays fast."""

import json
import subprocess
import sys

from tests.conftest import ROOT


def test_reference_arm_prints_one_contract_line():
    out = subprocess.run(
        [sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1",
         "--warmup", "1", "--cpu-sample-tokens", "128"],
        capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
                "cpu_baseline", "e2e", "impl"):
        assert key in d, key
    assert d["impl"] == "reference" and d["value"] > 0 and d["unit"] == "tokens/s"
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["config"]["workload"].startswith("cfg2")
    # the label names the sample actually timed, and the full config beside it
    assert d["config"]["tokens_per_gpu"] == 128
    assert d["config"]["full_config_tokens_per_gpu"] == 65536


def test_algorithmic_bytes_and_flops_of_the_benchmarked_configs():
    """The per-launch work the bench divides by kernel time: 18*H*I*k FLOPs
    per token over the six expert GEMMs, and each HBM kernel's tensors read or
    written once (cfg2: the gather reads x (128 MiB) and writes xs (1 GiB))."""
    sys.path.insert(0, str(ROOT))
    import bench
    c = bench.CONFIGS["cfg2"]
    T = c["T"]
    f = bench.gemm_flops(c, T)
    six = sum(v for n, v in f.items() if not n.startswith("router"))
    assert six == bench.layer_flops(c, T) == 18 * 1024 * 256 * 8 * T
    b = bench.hbm_bytes(c, T)
    assert b["gather"] == T * 1024 * 2 * (1 + 8)
    assert b["gather_bwd"] == T * 1024 * 2 * (8 + 2)
    for name in ("cfg3", "cfg4", "cfg5"):
        assert bench.CONFIG_INDEX[name] in (2, 3, 4)
