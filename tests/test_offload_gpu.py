"""load_and_offload on a small GPT-OSS configuration: every MoE block runs on
the QuantMoE path and equals the Hugging Face block computed on the same
(MXFP4-dequantised) expert weights; the whole model runs a forward pass and a
short greedy generation."""
from __future__ import annotations

import pytest
import torch

from tests.helpers import oracle_dequant, rel_l2
from tinyserve_b200.formats import TSB_MXFP4

pytestmark = pytest.mark.gpu


def _cfg():
    from transformers import GptOssConfig
    return GptOssConfig(hidden_size=512, intermediate_size=256, num_hidden_layers=2, num_local_experts=8,
                        num_experts_per_tok=2, num_attention_heads=8, num_key_value_heads=2, head_dim=64,
                        vocab_size=512, layer_types=["sliding_attention", "full_attention"])


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("CUDA required")
    return torch.device("cuda:0")


def test_moe_blocks_match_hf_block_on_dequantised_weights(dev):
    from transformers import GptOssForCausalLM
    from tinyserve_b200.offload import load_and_offload
    lm = load_and_offload(_cfg(), device="cuda", seed=5)
    assert len(lm.moe_layers) == 2 and all(q.packed for q in lm.moe_layers)
    torch.manual_seed(5)
    with dev:
        ref = GptOssForCausalLM(_cfg()).to(torch.bfloat16)  # the same seeded weights
    H, I = 512, 256
    for li, q in enumerate(lm.moe_layers):
        mlp = ref.model.layers[li].mlp
        with torch.no_grad():
            for e, ex in enumerate(q.experts):
                gu = torch.from_numpy(oracle_dequant(TSB_MXFP4, ex.gate.cpu(), ex.gate_scales.cpu(), 2 * I, H))
                dn = torch.from_numpy(oracle_dequant(TSB_MXFP4, ex.down.cpu(), ex.down_scales.cpu(), H, I))
                mlp.experts.gate_up_proj[e].copy_(gu.t())
                mlp.experts.down_proj[e].copy_(dn.t())
            mlp.float()
            x = torch.randn(1, 6, H, generator=torch.Generator().manual_seed(li)).to(dev)
            want, _ = mlp(x)
            got, w = lm.model.model.layers[li].mlp(x.to(torch.bfloat16))
        assert got.shape == want.shape and w.shape == (6, 2)
        # bf16 input and output rounding, bf16 router weights
        assert rel_l2(got.float().cpu().numpy(), want.float().cpu().numpy()) < 1e-2


def test_forward_and_generate(dev):
    from tinyserve_b200.offload import load_and_offload
    lm = load_and_offload(_cfg(), device="cuda", seed=7)
    ids = torch.randint(0, 512, (1, 5), generator=torch.Generator().manual_seed(3)).to(dev)
    with torch.no_grad():
        logits = lm(input_ids=ids).logits
    assert logits.shape == (1, 5, 512) and torch.isfinite(logits).all()
    out = lm.generate(input_ids=ids, max_new_tokens=4, do_sample=False)
    assert out.shape == (1, 9)
    assert all(q.device_error() == 0 for q in lm.moe_layers)
