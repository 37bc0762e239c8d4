"""The reference's own engines driving this build's quantized modules.

The reference integrates quantization by module replacement: its engines
look every projection up on its parent module at call time
(src/engine/paged_engine.py:98-105, graphed_decode_engine.py:81-110,
continuous_batching_engine.py:57-90), so swapping in QuantizedLinearInt8/Int4
must leave them working unchanged.  These tests run the unmodified engines —
BaselineEngine (HF forward with a KV cache), PagedEngine.generate,
ContinuousBatchingEngine.decode_step_batched and
GraphedDecodeEngine.decode_step_graphed (a CUDA graph captured around our
kernels) — on a random-init Qwen2 with Qwen2.5-1.5B's per-layer shapes,
quantized by quantize_model_int8 / quantize_model_int4, and compare every
greedy token with the same model whose quantized modules run the reference's
PyTorch path (w{8,4}a16_reference: dequantize to fp32, fp32 linear, cast).

Tokens must agree exactly.  The one tolerated difference is a near-tie: at
the first step where they differ, the reference path's two best logits must
lie closer together than the two paths' logits differ (kernel and oracle are
both within the fp16 output tolerance, so such a step can go either way);
the comparison stops there, since the sequences then diverge.  The CUDA-graph
engine must reproduce the eager PagedEngine's tokens on our kernels exactly.

The reference is imported from baseline/_ref (installed by
oracle/install_reference.py); the tests skip when it is not installed.
"""
import sys
from pathlib import Path

import pytest
import torch

from qlinear.quantization.int4 import quantize_model_int4
from qlinear.quantization.int8 import quantize_model_int8

from test_model_integration import _ReferencePath, _model

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="requires a CUDA GPU")]

REF = Path(__file__).resolve().parent.parent / "baseline" / "_ref"
VOCAB = 8192
BLOCK = 16


def _engines():
    if not (REF / "src" / "engine" / "paged_engine.py").exists():
        pytest.skip("the reference is not installed under baseline/_ref (oracle/install_reference.py)")
    sys.dont_write_bytecode = True
    if str(REF) not in sys.path:
        sys.path.append(str(REF))
    try:
        from src.engine.baseline_engine import BaselineEngine
        from src.engine.continuous_batching_engine import ContinuousBatchingEngine
        from src.engine.graphed_decode_engine import GraphedDecodeEngine
        from src.engine.paged_engine import PagedEngine
        from src.kv_cache.block_manager import PagedKVCacheManager
    except Exception as e:          # noqa: BLE001 - the skip reason names it
        pytest.skip(f"the reference's engines do not import here: {type(e).__name__}: {e}")
    return BaselineEngine, PagedEngine, ContinuousBatchingEngine, GraphedDecodeEngine, PagedKVCacheManager


class _Recorder(torch.nn.Module):
    """Wraps the lm_head and keeps a copy of the last-position logits of
    every call (what the engines take the argmax of)."""

    def __init__(self, head):
        super().__init__()
        self.head = head
        self.logits = []

    def forward(self, h):
        y = self.head(h)
        self.logits.append(y[:, -1, :].float().clone())
        return y


def _quantized_model(wbits):
    model = _model()
    stats = (quantize_model_int8 if wbits == 8 else quantize_model_int4)(model)
    assert stats["layers_quantized"] == 2 * 7
    model.lm_head = _Recorder(model.lm_head)
    return model


def _manager(PagedKVCacheManager, model, max_pages=64):
    cfg = model.config
    return PagedKVCacheManager(num_layers=cfg.num_hidden_layers, num_kv_heads=cfg.num_key_value_heads,
                               head_dim=cfg.hidden_size // cfg.num_attention_heads, block_size=BLOCK,
                               max_pages=max_pages, device="cuda", dtype=torch.float16)


def _prompt(n, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, VOCAB, (1, n), generator=g).cuda()


def _compare(ours, ref, logits_ours, logits_ref, what):
    """Token-exact agreement up to a near-tie (see the module docstring)."""
    assert len(ours) == len(ref) == len(logits_ours) == len(logits_ref), what
    for i, (a, b, la, lb) in enumerate(zip(ours, ref, logits_ours, logits_ref)):
        cos = torch.nn.functional.cosine_similarity(la.flatten(), lb.flatten(), dim=0).item()
        assert cos > 0.9999, f"{what}: step {i} logits cosine {cos}"
        if a == b:
            continue
        diff = (la - lb).abs().max().item()
        top2 = lb.flatten().topk(2).values
        gap = (top2[0] - top2[1]).item()
        assert gap <= 2 * diff, (f"{what}: step {i} token {a} vs reference {b}, not a near-tie "
                                 f"(reference top-2 gap {gap:.4g}, logits differ by {diff:.4g})")
        return i
    return len(ours)


@pytest.mark.parametrize("wbits", [8, 4])
def test_baseline_engine(wbits):
    BaselineEngine, *_ = _engines()
    model = _quantized_model(wbits)
    ids = _prompt(24, seed=3)

    def run():
        model.lm_head.logits.clear()
        eng = BaselineEngine(model, None, device="cuda")
        past, tok = eng.prefill(ids)
        toks = [tok.item()]
        for _ in range(7):
            past, tok = eng.decode_step(tok, past)
            toks.append(tok.item())
        return toks, list(model.lm_head.logits)

    ours, lo = run()
    with _ReferencePath(model):
        ref, lr = run()
    _compare(ours, ref, lo, lr, f"BaselineEngine w{wbits}")


@pytest.mark.parametrize("wbits", [8, 4])
def test_paged_engine_generate(wbits):
    _, PagedEngine, _, _, Manager = _engines()
    model = _quantized_model(wbits)
    ids = _prompt(40, seed=5)

    def run():
        model.lm_head.logits.clear()
        eng = PagedEngine(model, None, _manager(Manager, model), device="cuda")
        out = eng.generate(ids, max_new_tokens=10, seq_id=0)
        return out[0, ids.shape[1]:].tolist(), list(model.lm_head.logits)

    ours, lo = run()
    with _ReferencePath(model):
        ref, lr = run()
    _compare(ours, ref, lo, lr, f"PagedEngine w{wbits}")


@pytest.mark.parametrize("wbits", [8, 4])
def test_continuous_batching_engine(wbits):
    """Three sequences with different prompt lengths decoded together:
    batched M = 3 projections (decode kernel), per-sequence paged attention."""
    _, _, CBEngine, _, Manager = _engines()
    model = _quantized_model(wbits)
    prompts = {0: _prompt(9, seed=7), 1: _prompt(23, seed=8), 2: _prompt(40, seed=9)}

    def run():
        eng = CBEngine(model, None, _manager(Manager, model), device="cuda")
        cur = {sid: eng.prefill(p, sid) for sid, p in prompts.items()}
        model.lm_head.logits.clear()
        toks = []
        for _ in range(6):
            cur = eng.decode_step_batched(cur)
            toks.append([cur[sid].item() for sid in prompts])
        rows = [l for l in model.lm_head.logits]      # each (3, vocab)
        return toks, rows

    ours, lo = run()
    with _ReferencePath(model):
        ref, lr = run()
    for s in range(len(prompts)):
        _compare([t[s] for t in ours], [t[s] for t in ref], [l[s] for l in lo], [l[s] for l in lr],
                 f"ContinuousBatchingEngine w{wbits} sequence {s}")


@pytest.mark.parametrize("wbits", [8, 4])
def test_graphed_decode_engine(wbits):
    """decode_step_graphed captures the whole decode step — our kernels
    included — into a CUDA graph and replays it; the tokens must equal the
    eager PagedEngine's on the same kernels, and the reference path's."""
    _, PagedEngine, _, Graphed, Manager = _engines()
    model = _quantized_model(wbits)
    ids = _prompt(33, seed=11)

    eng = Graphed(model, None, _manager(Manager, model), max_context_len=256, device="cuda")
    graphed = eng.generate_graphed(ids, max_new_tokens=10, seq_id=0)[0, ids.shape[1]:].tolist()
    model.lm_head.logits.clear()
    eager_eng = PagedEngine(model, None, _manager(Manager, model), device="cuda")
    eager = eager_eng.generate(ids, max_new_tokens=10, seq_id=0)[0, ids.shape[1]:].tolist()
    lo = list(model.lm_head.logits)
    assert graphed == eager, (graphed, eager)

    model.lm_head.logits.clear()
    with _ReferencePath(model):
        ref_eng = PagedEngine(model, None, _manager(Manager, model), device="cuda")
        ref = ref_eng.generate(ids, max_new_tokens=10, seq_id=0)[0, ids.shape[1]:].tolist()
    _compare(eager, ref, lo, list(model.lm_head.logits), f"GraphedDecodeEngine w{wbits}")
    from qlinear import _lib
    assert _lib.device_error() == 0
