"""Loading one MoE layer of a Hugging Face Qwen3-MoE-style checkpoint into the
drop-in modules (CPU only: the loader copies tensors, it launches nothing)."""

import pytest
import torch

from moe_inference_verify_microbench_b200 import PermutedSparseMoE, load_qwen3_moe_layer
from moe_inference_verify_microbench_b200.ep import EPSparseMoELean, EPSparseMoEPure

H, I, E, K, LAYER = 64, 32, 8, 2, 3
PRE = f"model.layers.{LAYER}.mlp."


def _state_dict(seed=0):
    g = torch.Generator().manual_seed(seed)
    r = lambda *s: torch.randn(*s, generator=g).to(torch.bfloat16)  # noqa: E731
    sd = {PRE + "gate.weight": r(E, H), f"model.layers.{LAYER + 1}.mlp.gate.weight": r(E, H)}
    for e in range(E):
        sd[PRE + f"experts.{e}.gate_proj.weight"] = r(I, H)
        sd[PRE + f"experts.{e}.up_proj.weight"] = r(I, H)
        sd[PRE + f"experts.{e}.down_proj.weight"] = r(H, I)
    return sd


def _expert(sd, e, name):
    return sd[PRE + f"experts.{e}.{name}_proj.weight"]


def test_all_experts_into_the_stacked_bank():
    sd = _state_dict()
    mod = PermutedSparseMoE(H, I, E, K).to(torch.bfloat16)
    load_qwen3_moe_layer(mod, sd, LAYER)
    wg, wu, wd = mod.pack()
    assert torch.equal(mod.gate.weight, sd[PRE + "gate.weight"])
    for e in range(E):
        assert torch.equal(wg[e], _expert(sd, e, "gate"))
        assert torch.equal(wu[e], _expert(sd, e, "up"))
        assert torch.equal(wd[e], _expert(sd, e, "down"))
        # the per-expert parameters are views of the stack: one copy of the weights
        assert mod.experts[e].down_proj.weight.data_ptr() == wd[e].data_ptr()


@pytest.mark.parametrize("cls", [EPSparseMoELean, EPSparseMoEPure])
def test_expert_shard_into_an_ep_rank(cls):
    sd = _state_dict(1)
    mod = cls(H, I, E, K, 2, 1, group=None).to(torch.bfloat16)  # rank 1 owns experts 4..7
    load_qwen3_moe_layer(mod, sd, LAYER)
    wg, wu, wd = mod.pack()
    assert torch.equal(mod.gate.weight, sd[PRE + "gate.weight"])
    for local in range(E // 2):
        assert torch.equal(wg[local], _expert(sd, E // 2 + local, "gate"))
        assert torch.equal(wu[local], _expert(sd, E // 2 + local, "up"))
        assert torch.equal(wd[local], _expert(sd, E // 2 + local, "down"))


def test_missing_tensor_and_wrong_shape_are_reported_before_copying():
    sd = _state_dict(2)
    mod = PermutedSparseMoE(H, I, E, K).to(torch.bfloat16)
    before = mod.gate.weight.clone()
    bad = dict(sd)
    del bad[PRE + "experts.5.up_proj.weight"]
    with pytest.raises(KeyError, match="experts.5.up_proj"):
        load_qwen3_moe_layer(mod, bad, LAYER)
    bad = dict(sd)
    bad[PRE + "experts.2.down_proj.weight"] = torch.zeros(I, H, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="experts.2.down_proj"):
        load_qwen3_moe_layer(mod, bad, LAYER)
    assert torch.equal(mod.gate.weight, before)
    with pytest.raises(KeyError, match="layers.7"):
        load_qwen3_moe_layer(mod, sd, 7)
