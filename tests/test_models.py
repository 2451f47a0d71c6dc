"""The benchmark workloads are the reference's models (CPU, no GPU).

The harness builds its GPT, LLaMA and VGG16 clients itself
(kernel_intercept_b200/harness.py); these tests check that each issues the
same sequence of aten operators as the reference's own model code
(python/GPT.py CharGPT, python/LLaMA.py CharLLaMA, python/VGG16.py
VGG16Model) at small sizes: the forward in eval mode, and for the GPT a
training step (forward, cross-entropy, backward) as the BE clients run it.
The captured dense ops are a subset of these operators, so equal sequences
mean the interposer sees the same calls from either model.

The reference files come from baseline/_ref/python (copied there unmodified
by ``make -C oracle ref-drivers REF=<reference checkout>``); the tests are
skipped when they are absent.
"""
import importlib
import os
import sys

import pytest
import torch
from torch.utils._python_dispatch import TorchDispatchMode

from kernel_intercept_b200 import harness

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
DRIVERS = os.path.join(ROOT, "baseline", "_ref", "python")


def _ref_module(name):
    if not os.path.exists(os.path.join(DRIVERS, name + ".py")):
        pytest.skip("reference drivers not staged (make -C oracle ref-drivers REF=...)")
    if DRIVERS not in sys.path:
        sys.path.insert(0, DRIVERS)
    return importlib.import_module(name)


class _OpLog(TorchDispatchMode):
    def __init__(self):
        super().__init__()
        self.ops = []

    def __torch_dispatch__(self, func, types, args=(), kwargs=None):
        self.ops.append(str(func.overloadpacket))
        return func(*args, **(kwargs or {}))


def _ops(fn):
    with _OpLog() as log:
        fn()
    return log.ops


def test_gpt_matches_reference_model():
    ref = _ref_module("GPT")
    emb, head, layers, seq, vocab = 64, 16, 2, 32, 100
    ref.emb_size, ref.head_size, ref.n_layer, ref.sequence_len = emb, head, layers, seq
    theirs = ref.CharGPT(vocab)
    ours = harness.make_gpt(vocab=vocab, emb=emb, head_size=head, layers=layers, seq=seq,
                            device="cpu")
    assert [type(m).__name__ for m in theirs.modules()].count("Linear") == \
        [type(m).__name__ for m in ours.modules()].count("Linear")
    tok = torch.randint(0, vocab, (2, seq))
    tgt = torch.randint(0, vocab, (2, seq))

    def train(m):
        def step():
            m.train()
            logits = m(tok)
            loss = torch.nn.functional.cross_entropy(logits.view(-1, vocab), tgt.view(-1))
            loss.backward()
        return step

    def infer(m):
        def step():
            m.eval()
            with torch.no_grad():
                m(tok)
        return step

    assert _ops(infer(ours)) == _ops(infer(theirs))
    assert _ops(train(ours)) == _ops(train(theirs))


def test_llama_matches_reference_model():
    ref = _ref_module("LLaMA")
    hidden, heads, layers, inter, seq, vocab = 64, 4, 2, 96, 32, 100
    ref.hidden_size, ref.num_heads, ref.num_kv_heads = hidden, heads, heads
    ref.num_layers, ref.intermediate_size, ref.sequence_len = layers, inter, seq
    ref.rms_norm_eps, ref.rope_theta = 1e-6, 1e4
    theirs = ref.CharLLaMA(vocab).to(torch.bfloat16).eval()
    ours = harness.make_llama(vocab=vocab, hidden=hidden, heads=heads, layers=layers,
                              inter=inter, seq=seq, device="cpu",
                              dtype=torch.bfloat16).eval()
    tok = torch.randint(0, vocab, (2, seq))

    def infer(m):
        def step():
            with torch.no_grad():
                m(tok)
        return step

    assert _ops(infer(ours)) == _ops(infer(theirs))


def test_vgg16_matches_reference_model():
    ref = _ref_module("VGG16")
    theirs = ref.VGG16Model().eval()
    ours = harness.make_vgg16("cpu").eval()
    x = torch.randn(1, 3, 64, 64)

    def infer(m):
        def step():
            with torch.no_grad():
                m(x)
        return step

    assert _ops(infer(ours)) == _ops(infer(theirs))
