"""GPU runs of the decode step and the local head on weights read through the
ONNX reader (mockbird_b200.onnx_weights) from a synthetic model in the layout of
the published graphs (tests/golden/make_onnx_fixture.py: hidden 64, FFN 256, 2
layers, 16 codebooks of 128 codes), through the C ABI, against the CPU oracle
on the same weight arrays (max-abs 2e-2, the decoder tests' tolerance)."""
import os
import sys

import numpy as np
import pytest
import torch

import oracle
from gpu_util import max_err
from mockbird_b200 import KvRing, LocalHead
from mockbird_b200.engine import Decoder
from mockbird_b200.onnx_weights import decoder_weights, local_head_weights, open_model

sys.path.insert(0, os.path.join(os.path.dirname(__file__), "golden"))
import make_onnx_fixture as fx  # noqa: E402

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
TOL = 2e-2


@pytest.fixture(scope="module")
def tables(tmp_path_factory):
    d = str(tmp_path_factory.mktemp("onnx"))
    fx.write_fixture(d)
    return (open_model(os.path.join(d, "global.onnx"), os.path.join(d, "global.data")),
            open_model(os.path.join(d, "local.onnx"), os.path.join(d, "local.data")))


def test_decoder_step_on_onnx_weights(tables):
    g, _ = tables
    w = decoder_weights(g, layers=fx.LAYERS, hidden=fx.HIDDEN, ffn=fx.FFN)
    heads = fx.HIDDEN // 64
    ring = KvRing(layers=fx.LAYERS, heads=heads, streams=3, capacity=64, dtype="bf16", wrap=True)
    dec = Decoder(ring, w, fx.FFN)
    orc = oracle.Ring(layers=fx.LAYERS, streams=3, heads=heads, capacity=64, dtype="bf16", wrap=True)
    rng = np.random.default_rng(1)
    worst = 0.0
    for step in range(12):
        x = rng.standard_normal((3, fx.HIDDEN)).astype(np.float32)
        pos = [step, step + 2, step + 5]
        got = dec.step([2, 0, 1], pos, torch.from_numpy(x).to(DEV))
        want = oracle.decoder_step(orc, w, fx.FFN, [2, 0, 1], pos, x)
        worst = max(worst, max_err(got, want))
    ring.sync()
    dec.dispose()
    assert worst < TOL, worst


def test_local_head_frame_on_onnx_weights(tables):
    g, loc = tables
    channels = 16
    w = local_head_weights(loc, g, fx.ASSISTANT_SLOT, fx.AUDIO_END, hidden=fx.HIDDEN, ffn=fx.FFN, codes=fx.CODES,
                           channels=channels)
    heads = fx.HIDDEN // 64
    ring = KvRing(layers=1, heads=heads, streams=2, capacity=channels + 1, dtype="f32", wrap=False,
                  max_position=channels + 1)
    head = LocalHead(ring, w, fx.FFN, fx.CODES, channels, 1.2)
    x = np.random.default_rng(2).standard_normal((2, fx.HIDDEN)).astype(np.float32)
    tok, cont, lg = head.frame([1, 0], torch.from_numpy(x).to(DEV), logits=True)
    tok, lg = tok.cpu().numpy(), lg.cpu().numpy()
    orc = oracle.Ring(layers=1, streams=2, heads=heads, capacity=channels + 1, dtype="f32", wrap=False,
                      max_position=channels + 1)
    seen = np.zeros((2, channels, fx.CODES // 32), np.uint32)
    _, cont_o, lg_o, _ = oracle.local_frame(orc, w, fx.FFN, fx.CODES, channels, 1.2, [1, 0], x, seen, forced=tok)
    assert max_err(lg, lg_o) < TOL
    # each pick is the argmax of the kernel's own logits (the seen masks are per
    # channel, so the first frame after a clear penalises nothing)
    fresh = np.zeros(fx.CODES // 32, np.uint32)
    assert all(tok[i, c] == oracle.argmax_penalty(lg[i, c], fresh, 1.2) for i in range(2) for c in range(channels))
    ring.sync()
    head.dispose()
