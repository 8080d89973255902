"""Whole-model GPT-OSS decode (tinyserve_b200.gptoss.GptOssDecoder) on a small
configuration against the Hugging Face model computed in fp32 on the same
weights (experts = the MXFP4-dequantised weights the QuantMoE layers hold):
prefill logits, then CUDA-graph decode steps, with a bf16 and an FP8 (e4m3)
KV cache; sliding-window layers with a window shorter than the prompt."""
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
                        vocab_size=512, sliding_window=4, layer_types=["sliding_attention", "full_attention"])


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("CUDA required")
    return torch.device("cuda:0")


def _reference(lm, dev):
    """HF model in fp32 with the same seeded dense weights and the QuantMoE
    layers' dequantised experts."""
    from transformers import GptOssForCausalLM
    torch.manual_seed(11)
    with dev:
        ref = GptOssForCausalLM(_cfg()).to(torch.bfloat16)
    H, I = 512, 256
    with torch.no_grad():
        for li, q in enumerate(lm.moe_layers):
            mlp = ref.model.layers[li].mlp
            for e, ex in enumerate(q.experts):
                gu = torch.from_numpy(oracle_dequant(TSB_MXFP4, ex.gate.cpu(), ex.gate_scales.cpu(), 2 * I, H))
                dn = torch.from_numpy(oracle_dequant(TSB_MXFP4, ex.down.cpu(), ex.down_scales.cpu(), H, I))
                mlp.experts.gate_up_proj[e].copy_(gu.t())
                mlp.experts.down_proj[e].copy_(dn.t())
    ref.float()
    ref.config._attn_implementation = "eager"
    return ref.eval()


@pytest.mark.parametrize("kv", ["bf16", "fp8"])
def test_decoder_matches_hf_fp32(dev, kv):
    from tinyserve_b200.gptoss import GptOssDecoder
    from tinyserve_b200.offload import load_and_offload
    lm = load_and_offload(_cfg(), device="cuda", seed=11)
    ref = _reference(lm, dev)
    kv_dtype = torch.bfloat16 if kv == "bf16" else torch.float8_e4m3fn
    dec = GptOssDecoder(lm.model, lm.moe_layers, max_seq=64, kv_dtype=kv_dtype, prefill_chunk=4)
    tol = 2e-2 if kv == "bf16" else 6e-2
    prompt = torch.randint(0, 512, (10,), generator=torch.Generator().manual_seed(3)).to(dev)
    logits = dec.prefill(prompt)
    with torch.no_grad():
        want = ref(input_ids=prompt[None]).logits[0, -1].float()
    assert rel_l2(logits.cpu().numpy(), want.cpu().numpy()) < tol
    seq = prompt.clone()
    tok = logits.argmax().reshape(1)
    for _ in range(4):
        seq = torch.cat([seq, tok])
        nxt = dec.step(tok)
        got = dec._logits[0].float()
        with torch.no_grad():
            want = ref(input_ids=seq[None]).logits[0, -1].float()
        assert rel_l2(got.cpu().numpy(), want.cpu().numpy()) < tol
        assert int(nxt) == int(got.argmax())
        tok = nxt.clone()
    assert dec.length == 14
    assert all(q.device_error() == 0 for q in lm.moe_layers)


def test_generate_runs_past_the_window(dev):
    from tinyserve_b200.gptoss import GptOssDecoder
    from tinyserve_b200.offload import load_and_offload
    lm = load_and_offload(_cfg(), device="cuda", seed=12)
    dec = GptOssDecoder(lm.model, lm.moe_layers, max_seq=40)
    prompt = torch.randint(0, 512, (7,), generator=torch.Generator().manual_seed(4)).to(dev)
    out = dec.generate(prompt, 12)
    assert out.shape == (12,) and int(out.min()) >= 0 and int(out.max()) < 512
    assert dec.length == 7 + 11
