"""GPU parity of the decode step around the path (BASELINE config 4 shape):
LayerNorm, QKV/c_proj/fc_in/fc_out GEMMs (bf16 weights), GELU(tanh), residuals,
ln_f, and the fused append + attention, against the CPU oracle."""
import numpy as np
import pytest
import torch

import oracle
from gpu_util import max_err
from mockbird_b200 import KvRing, MockbirdError
from mockbird_b200.engine import Decoder

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
TOL = 2e-2  # bf16 weights and GEMM inputs, 12-head attention over bf16 storage, accumulated over the layers


def _weights(layers, h, ffn, seed):
    n = Decoder.weight_count(layers, h, ffn)
    w = (np.random.default_rng(seed).standard_normal(n) * 0.02).astype(np.float32)
    # LayerNorm gains at 1 (the published model's LN scales are all ones) and biases small
    off = 0
    per = 2 * h + h * 3 * h + 3 * h + h * h + h + 2 * h + h * ffn + ffn + ffn * h + h
    for l in range(layers):
        base = l * per
        w[base:base + h] = 1.0
        w[base + 2 * h + h * 3 * h + 3 * h + h * h + h: base + 2 * h + h * 3 * h + 3 * h + h * h + 2 * h] = 1.0
    w[layers * per: layers * per + h] = 1.0
    return w


@pytest.mark.parametrize("dtype,layers,ffn", [("bf16", 2, 3072), ("f32", 1, 1024), ("f16", 1, 1024)])
def test_decoder_step_matches_oracle(dtype, layers, ffn):
    h, S, C = 768, 5, 256
    w = _weights(layers, h, ffn, seed=layers)
    ring = KvRing(layers=layers, streams=S, capacity=C, dtype=dtype, wrap=True)
    dec = Decoder(ring, w, ffn)
    orc = oracle.Ring(layers=layers, streams=S, heads=12, capacity=C, dtype=dtype, wrap=True)
    rng = np.random.default_rng(3)
    order = [4, 1, 0, 3]
    worst = 0.0
    for step in range(40):
        x = rng.standard_normal((len(order), h)).astype(np.float32)
        pos = [step + 7 * i for i in range(len(order))]  # different positions per stream
        got = dec.step(order, pos, torch.from_numpy(x).to(DEV))
        ref = oracle.decoder_step(orc, w, ffn, order, pos, x)
        worst = max(worst, max_err(got, ref))
    ring.sync()
    assert worst < TOL, worst
    # the K/V rows that the QKV GEMM's epilogue roped and appended: the windows
    # hold the same positions in the same order as the oracle's ring, and the rows
    # agree within the step's tolerance (the GEMM sums in another order)
    for layer in range(layers):
        for i, s in enumerate(order):
            k, v, slots = ring.gather(layer, s, 39 + 7 * i)
            ok, ov, oslots = orc.gather(layer, s, 39 + 7 * i)
            assert np.array_equal(slots.cpu().numpy(), oslots), (layer, s)
            for got_rows, want_bits in ((k, ok), (v, ov)):
                want = {"f32": lambda b: b, "bf16": lambda b: (b.astype(np.uint32) << 16).view(np.float32),
                        "f16": lambda b: b.view(np.float16).astype(np.float32)}[dtype](want_bits)
                assert np.abs(got_rows.float().cpu().numpy() - want).max() < TOL, (layer, s)


def test_decoder_rejects_bad_weights():
    ring = KvRing(layers=1, streams=2, capacity=64, dtype="bf16", wrap=True)
    with pytest.raises(ValueError):
        Decoder(ring, np.zeros(10, np.float32), 3072)
    dec = Decoder(ring, _weights(1, 768, 1024, 0), 1024)
    with pytest.raises(MockbirdError):
        dec.step([0, 1, 0], [0, 0, 0], torch.zeros(3, 768, device=DEV))  # 3 items > max_batch 2


def test_decoder_step_host_matches_device_step():
    """mb_decoder_step_host (host rows in, ln_f rows out, one synchronisation: the
    call globalStep makes) equals mb_decoder_step on device arrays bit for bit,
    step after step, over rings that start equal -- the first step of the batch
    size runs directly, the later ones replay the captured step."""
    h, S, C, layers, ffn = 768, 6, 128, 2, 1024
    w = _weights(layers, h, ffn, seed=9)
    ra = KvRing(layers=layers, streams=S, capacity=C, dtype="bf16", wrap=True)
    rb = KvRing(layers=layers, streams=S, capacity=C, dtype="bf16", wrap=True)
    da, db = Decoder(ra, w, ffn), Decoder(rb, w, ffn)
    rng = np.random.default_rng(11)
    order = [5, 0, 3, 1]
    pinned = torch.empty(len(order), h).pin_memory()
    for step in range(6):
        x = rng.standard_normal((len(order), h)).astype(np.float32)
        pos = [step + 3 * i for i in range(len(order))]
        dev = db.step(order, pos, torch.from_numpy(x).to(DEV)).cpu().numpy()
        if step % 2:  # a pinned tensor and a plain numpy array both work
            pinned.copy_(torch.from_numpy(x))
            host = da.step_host(order, pos, pinned).numpy()
        else:
            host = da.step_host(order, pos, x.copy())
        assert np.array_equal(host, dev), step
    ra.sync()
    rb.sync()


def test_decoder_step_host_checks_items_on_the_host():
    ring = KvRing(layers=1, streams=3, capacity=64, dtype="bf16", wrap=True)
    dec = Decoder(ring, _weights(1, 768, 1024, 0), 1024)
    x = np.zeros((2, 768), np.float32)
    with pytest.raises(MockbirdError, match="twice"):
        dec.step_host([1, 1], [0, 0], x)
    with pytest.raises(MockbirdError, match="out of range"):
        dec.step_host([0, 3], [0, 0], x)
    with pytest.raises(MockbirdError, match="position"):
        dec.step_host([0, 1], [0, -1], x)
    with pytest.raises(TypeError):
        dec.step_host([0, 1], [0, 0], np.zeros((2, 700), np.float32))
    # the context still works after the rejections
    out = dec.step_host([0, 1], [0, 0], np.ones((2, 768), np.float32))
    assert np.isfinite(out).all()
    ring.sync()


def test_decoder_step_at_config4_shape():
    """BASELINE config 4's shape: 256 streams through all 12 layers (hidden 768,
    FFN 3072, bf16 ring of 2048 slots), positions U[444, 2048) from seed 0, every
    window filled with N(0,1) K/V, two steps.  The oracle tracks 8 of the streams
    (a host ring for all 256 would take 19 GB): their rows match within the
    decoder tolerance and their windows (the appended rows included) keep the
    oracle's slot order, while the other 248 streams load the GEMMs and the
    decode kernel as the bench does."""
    h, ffn, L, S, C = 768, 3072, 12, 256, 2048
    w = _weights(L, h, ffn, seed=4)
    ring = KvRing(layers=L, streams=S, capacity=C, dtype="bf16", wrap=True)
    dec = Decoder(ring, w, ffn)
    track = [0, 12, 37, 64, 101, 128, 200, 255]
    orc = oracle.Ring(layers=L, streams=len(track), heads=12, capacity=C, dtype="bf16", wrap=True)
    pos = np.random.default_rng(0).integers(444, 2048, size=S)
    gen = torch.Generator(device=DEV)
    gen.manual_seed(4)
    for s in range(S):
        p = int(pos[s])
        kv = torch.randn(2, 12, p, 64, generator=gen, device=DEV).to(torch.bfloat16)
        bits = kv.view(torch.int16).cpu().numpy().view(np.uint16) if s in track else None
        for layer in range(L):
            ring.ring_write(layer, s, 0, kv[0], kv[1])
            if bits is not None:
                i = track.index(s)
                orc.kv_view()[layer, i, :, :, :p] = bits
                orc.slot_pos[layer, i, :p] = np.arange(p, dtype=np.int32)
    rng = np.random.default_rng(5)
    worst = 0.0
    for step in range(2):
        x = rng.standard_normal((S, h)).astype(np.float32)
        p_now = pos + step
        got = dec.step(list(range(S)), p_now, torch.from_numpy(x).to(DEV)).cpu().numpy()
        ref = oracle.decoder_step(orc, w, ffn, list(range(len(track))), p_now[track], x[track])
        worst = max(worst, max_err(got[track], ref))
    ring.sync()
    assert worst < TOL, worst
    for i, s in enumerate(track):
        for layer in (0, L - 1):
            k, v, slots = ring.gather(layer, s, int(pos[s]) + 1)
            ok, ov, oslots = orc.gather(layer, i, int(pos[s]) + 1)
            assert np.array_equal(slots.cpu().numpy(), oslots), (layer, s)


@pytest.mark.parametrize("S", [256, 131])
def test_decoder_split_matches_one_chain(S, monkeypatch):
    """A step of 128 items or more runs as two half-batch chains on two CUDA
    streams, each over its own rows of the activations and of the split-K
    scratch.  The same two steps with the split off (MOCKBIRD_DECODER_SPLIT=0,
    read when the decoder is created) give every row within the decoder
    tolerance (the GEMMs' plans differ with M, so their sums may round
    differently).  The appended K/V rows land in the same slots.  131 items split
    65 + 66, so the second chain starts at a row that is not a tile boundary."""
    h, ffn, L, C = 768, 3072, 2, 1024
    w = _weights(L, h, ffn, seed=6)
    rings, decs = [], []
    for split in ("1", "0"):
        monkeypatch.setenv("MOCKBIRD_DECODER_SPLIT", split)
        ring = KvRing(layers=L, streams=S, capacity=C, dtype="bf16", wrap=True)
        rings.append(ring)
        decs.append(Decoder(ring, w, ffn))
    monkeypatch.delenv("MOCKBIRD_DECODER_SPLIT")
    pos = np.random.default_rng(7).integers(300, C, size=S)
    gen = torch.Generator(device=DEV)
    gen.manual_seed(7)
    for s in range(S):
        kv = torch.randn(2, 12, int(pos[s]), 64, generator=gen, device=DEV).to(torch.bfloat16)
        for layer in range(L):
            for ring in rings:
                ring.ring_write(layer, s, 0, kv[0], kv[1])
    rng = np.random.default_rng(8)
    worst = 0.0
    for step in range(2):
        x = torch.from_numpy(rng.standard_normal((S, h)).astype(np.float32)).to(DEV)
        outs = [dec.step(list(range(S)), pos + step, x.clone()).cpu().numpy() for dec in decs]
        assert np.isfinite(outs[0]).all()
        worst = max(worst, max_err(outs[0], outs[1]))
    for ring in rings:
        ring.sync()
    assert worst < TOL, worst
    for s in (0, S // 2 - 1, S // 2, S // 2 + 1, S - 1):
        for layer in range(L):
            a = rings[0].gather(layer, s, int(pos[s]) + 1)
            b = rings[1].gather(layer, s, int(pos[s]) + 1)
            assert torch.equal(a[2], b[2]), (layer, s)
            assert (a[0].float() - b[0].float()).abs().max().item() < TOL, (layer, s)
    for dec in decs:
        dec.dispose()
    for ring in rings:
        ring.dispose()
