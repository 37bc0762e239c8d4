"""Model-level drop-in check on the GPU (replaces the reference's e2e tests,
tests/test_e2e_quantization.py:48-118 and tests/test_e2e_int4.py:56-110,
which need the Qwen2.5 checkpoint: no network here).

A random-init Qwen2 with Qwen2.5-1.5B's per-layer shapes (hidden 1536,
12 query / 2 KV heads, head_dim 128, intermediate 8960; 2 layers) is
quantized in place by quantize_model_int8 / quantize_model_int4, exactly as
the reference does.  Its outputs must match the same quantized model run
through the reference's own PyTorch path (w{8,4}a16_reference: dequantize to
fp32, fp32 linear, cast): prefill (64 tokens, tensor-core path) and greedy
decoding (M = 1, decode kernel) through HF's generate with a KV cache.
"""
import pytest
import torch

from qlinear.kernels.w4a16_matmul import w4a16_reference
from qlinear.kernels.w8a16_matmul import w8a16_reference
from qlinear.quantization.int4 import QuantizedLinearInt4, quantize_model_int4
from qlinear.quantization.int8 import QuantizedLinearInt8, quantize_model_int8

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="requires a CUDA GPU")]


def _model():
    from transformers import Qwen2Config, Qwen2ForCausalLM
    cfg = Qwen2Config(vocab_size=8192, hidden_size=1536, intermediate_size=8960, num_hidden_layers=2,
                      num_attention_heads=12, num_key_value_heads=2, max_position_embeddings=512,
                      tie_word_embeddings=False)
    torch.manual_seed(0)
    m = Qwen2ForCausalLM(cfg)
    with torch.no_grad():
        for p in m.parameters():
            p.normal_(0.0, 0.02)
    return m.half().cuda().eval()


class _ReferencePath:
    """Runs every quantized module through the reference's PyTorch oracle."""

    def __init__(self, model):
        self.mods = [mod for mod in model.modules() if isinstance(mod, (QuantizedLinearInt4, QuantizedLinearInt8))]
        self.saved = []

    def __enter__(self):
        for mod in self.mods:
            self.saved.append(mod.forward)
            if isinstance(mod, QuantizedLinearInt4):
                mod.forward = (lambda m: lambda x: w4a16_reference(x, m.weight_packed, m.scales, m.bias,
                                                                   layout=m.layout))(mod)
            else:
                mod.forward = (lambda m: lambda x: w8a16_reference(x, m.weight_q, m.scale, m.bias))(mod)
        return self

    def __exit__(self, *exc):
        for mod, f in zip(self.mods, self.saved):
            mod.forward = f
        return False


@pytest.mark.parametrize("wbits", [8, 4])
def test_quantized_model_matches_reference_path(wbits):
    model = _model()
    stats = (quantize_model_int8 if wbits == 8 else quantize_model_int4)(model)
    assert stats["layers_quantized"] == 2 * 7
    g = torch.Generator().manual_seed(1)
    ids = torch.randint(0, 8192, (1, 64), generator=g).cuda()
    with torch.no_grad():
        ours = model(ids).logits.float()
        with _ReferencePath(model):
            ref = model(ids).logits.float()
    cos = torch.nn.functional.cosine_similarity(ours.flatten(), ref.flatten(), dim=0).item()
    assert cos > 0.9999, cos
    agree = (ours.argmax(-1) == ref.argmax(-1)).float().mean().item()
    assert agree >= 0.98, agree
    # greedy decoding with a KV cache: prefill M = 64, then M = 1 steps
    with torch.no_grad():
        out = model.generate(ids[:, :16], max_new_tokens=8, do_sample=False)
        with _ReferencePath(model):
            out_ref = model.generate(ids[:, :16], max_new_tokens=8, do_sample=False)
    assert torch.equal(out, out_ref), (out.tolist(), out_ref.tolist())
    from qlinear import _lib
    assert _lib.device_error() == 0
