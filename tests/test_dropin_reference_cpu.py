"""Drop-in check against the reference's own training code (CPU, structure only).

The reference's ByteLM is built with sparse blocks and every block's mlp is
swapped for spark_gpt_b200.SparseMoE (the two-line edit a trainer makes).  The
reference's own build_optimizer (train.py:3056-3095), apply_mup_init
(:2718-2745) and export_unfused_state_dict (:2540-2558) must then see the same
tensors as with its own SparseMoE: the same parameter names, shapes and
dtypes, the same optimizer groups, the same init draws under one seed and the
same export keys.  The layer's forward needs a B200 and is covered by the GPU
tests.  The reference checkout is named by the SPARK_GPT_REFERENCE environment
variable (the directory holding its train.py); the test is skipped when the
variable is unset or the checkout is absent (it never travels to a GPU box).
"""

import os
import sys
from pathlib import Path
from types import SimpleNamespace

import pytest
import torch

REF_ENV = os.environ.get("SPARK_GPT_REFERENCE")
REF = Path(REF_ENV) if REF_ENV else None


@pytest.fixture(scope="module")
def train():
    if REF is None:
        pytest.skip("SPARK_GPT_REFERENCE is unset (path of the reference checkout)")
    if not (REF / "train.py").exists():
        pytest.skip("reference checkout not present")
    old = sys.dont_write_bytecode
    sys.dont_write_bytecode = True
    sys.path.insert(0, str(REF))
    try:
        import train as t  # the reference module, imported in place
    except ImportError as e:  # its import-time dependencies (flash-attn) are missing
        pytest.skip(f"reference not importable here: {e}")
    finally:
        sys.path.remove(str(REF))
        sys.dont_write_bytecode = old
    return t


def _models(train):
    from spark_gpt_b200 import SparseMoE
    cfg = train.ModelConfig(hidden_size=128, num_hidden_layers=3, intermediate_size=256,
                            num_attention_heads=2, num_key_value_heads=1, head_dim=64,
                            num_experts=8, num_experts_per_tok=2, moe_intermediate_size=64,
                            max_position_embeddings=64, mlp_only_layers=(1,))
    torch.manual_seed(0)
    ref = train.ByteLM(cfg)
    torch.manual_seed(0)
    ours = train.ByteLM(cfg)
    swapped = 0
    for block in ours.layers:
        if block.is_sparse:
            block.mlp = SparseMoE(cfg)
            swapped += 1
    assert swapped == 2  # layer 1 stays a dense MLP (mlp_only_layers)
    return cfg, ref, ours


def test_parameters_and_init_match_the_reference_model(train):
    cfg, ref, ours = _models(train)
    a = {n: (tuple(p.shape), p.dtype) for n, p in ref.named_parameters()}
    b = {n: (tuple(p.shape), p.dtype) for n, p in ours.named_parameters()}
    assert a == b
    for model in (ref, ours):
        torch.manual_seed(1)
        train.apply_mup_init(model, base_dim=64, emb_std=0.02, hidden_std=0.02)
    for (n, p), (_, q) in zip(ref.named_parameters(), ours.named_parameters()):
        assert torch.equal(p, q), n


def test_optimizer_groups_match_the_reference_model(train):
    cfg, ref, ours = _models(train)
    args = SimpleNamespace(mup_base_dim=64, model_dim=cfg.hidden_size, router_lr=None,
                           adamw_lr=1e-3, muon_lr=0.02, muon_momentum=0.95, weight_decay=0.0)
    groups = []
    for model in (ref, ours):
        opt, info = train.build_optimizer(model, args)
        names = {id(p): n for n, p in model.named_parameters()}
        groups.append(([sorted(names[id(p)] for p in g["params"]) for g in opt.param_groups],
                       info))
    assert groups[0] == groups[1]
    muon = groups[1][0][0]
    assert "layers.0.mlp.experts.gate_up_proj" in muon and "layers.2.mlp.experts.down_proj" in muon
    assert "layers.0.mlp.gate.weight" in groups[1][0][3]  # the router's no-decay AdamW group


def test_hf_export_keys_match_the_reference_model(train):
    cfg, ref, ours = _models(train)
    a = {k: tuple(v.shape) for k, v in train.export_unfused_state_dict(ref).items()}
    b = {k: tuple(v.shape) for k, v in train.export_unfused_state_dict(ours).items()}
    assert a == b
    assert a["layers.0.mlp.experts.gate_up_proj"] == (8, 128, 128)


def test_hf_export_of_the_swapped_model_strictly_loads_as_qwen3_moe(train, tmp_path):
    """The reference's export_hf (train.py:2614-2691) on the model with this
    layer swapped in writes a directory that transformers strictly loads as
    Qwen3MoeForCausalLM, with every tensor equal to the reference model's own
    export under the same init (the reference's tests/test_moe.py:260-290)."""
    transformers = pytest.importorskip("transformers")
    cfg, ref, ours = _models(train)
    for model in (ref, ours):
        torch.manual_seed(2)
        train.apply_mup_init(model, base_dim=64, emb_std=0.02, hidden_std=0.02)
    train.export_hf(ours, tmp_path)
    loaded = transformers.AutoModelForCausalLM.from_pretrained(tmp_path)
    assert loaded.__class__.__name__ == "Qwen3MoeForCausalLM"
    actual = loaded.state_dict()
    expected = {(k if k == "lm_head.weight" else "model." + k): v
                for k, v in train.export_unfused_state_dict(ref).items()}
    assert set(actual) == set(expected)
    for key, value in expected.items():
        torch.testing.assert_close(actual[key], value)
