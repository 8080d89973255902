"""Continuous-batching serving (tinyserve_b200.serving.ServingEngine) against
the batch-1 decoder on the same small GPT-OSS model: every emitted token's
logits equal (within bf16 GEMM-vs-GEMV rounding) those of GptOssDecoder fed
the same tokens, with more requests than cache slots (queueing and slot
reuse), different prompt lengths and a batch above 16 tokens (the grouped
expert path)."""
from __future__ import annotations

import pytest
import torch

from tests.helpers import rel_l2

pytestmark = pytest.mark.gpu


def _cfg():
    from transformers import GptOssConfig
    return GptOssConfig(hidden_size=512, intermediate_size=256, num_hidden_layers=2, num_local_experts=8,
                        num_experts_per_tok=2, num_attention_heads=8, num_key_value_heads=2, head_dim=64,
                        vocab_size=512, sliding_window=4, layer_types=["sliding_attention", "full_attention"])


@pytest.fixture(scope="module")
def lm():
    if not torch.cuda.is_available():
        pytest.skip("CUDA required")
    from tinyserve_b200.offload import load_and_offload
    return load_and_offload(_cfg(), device="cuda", seed=21)


def _check_against_decoder(lm, req, kv_dtype):
    from tinyserve_b200.gptoss import GptOssDecoder
    dec = GptOssDecoder(lm.model, lm.moe_layers, max_seq=64, kv_dtype=kv_dtype, prefill_chunk=4)
    got = dec.prefill(req.prompt.cuda())
    assert rel_l2(req.logits[0].numpy(), got.cpu().numpy()) < 1e-2
    for i in range(1, len(req.generated)):
        dec.step(req.generated[i - 1])
        assert rel_l2(req.logits[i].numpy(), dec._logits[0].float().cpu().numpy()) < 1e-2


@pytest.mark.parametrize("kv", ["bf16", "fp8"])
def test_serving_matches_single_request_decoder(lm, kv):
    from tinyserve_b200.serving import ServingEngine
    kv_dtype = torch.bfloat16 if kv == "bf16" else torch.float8_e4m3fn
    eng = ServingEngine(lm.model, lm.moe_layers, max_batch=2, max_seq=64, kv_dtype=kv_dtype, prefill_chunk=4,
                        keep_logits=True)
    g = torch.Generator().manual_seed(5)
    lens, news = (5, 9, 3), (6, 4, 7)
    ids = [eng.submit(torch.randint(0, 512, (n,), generator=g), m) for n, m in zip(lens, news)]
    out = eng.run()
    assert sorted(out) == ids and [len(out[i]) for i in ids] == list(news)
    for i in ids:
        _check_against_decoder(lm, eng.finished[i], kv_dtype)
    assert all(q.device_error(1) == 0 for q in lm.moe_layers)


def test_serving_batch_above_16(lm):
    """20 requests decoding together: the expert layer takes the grouped path."""
    from tinyserve_b200.serving import ServingEngine
    eng = ServingEngine(lm.model, lm.moe_layers, max_batch=20, max_seq=32, kv_dtype=torch.bfloat16,
                        prefill_chunk=8, keep_logits=True)
    g = torch.Generator().manual_seed(6)
    ids = [eng.submit(torch.randint(0, 512, (3 + i % 5,), generator=g), 3) for i in range(20)]
    assert eng.step() == 20  # all admitted and decoded together
    out = eng.run()
    assert sorted(out) == ids
    for i in (0, 7, 19):
        _check_against_decoder(lm, eng.finished[i], torch.bfloat16)
