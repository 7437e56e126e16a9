"""GPU parity of the local 17-step head (DecodeRunner.nextFrame, decode.ts:788-939)
and of ARGMAX_PENALTY (kernels-decode.ts:428-485) against the CPU oracle.

The head's picks feed its own next step, so a near-tie that the two sides break
differently (fp32 sums in another order) would make every later step differ.
The parity test therefore follows the kernel's picks in the oracle (teacher
forcing) and checks three things per step: the logits within tolerance, the
kernel's pick exactly equal to the penalised argmax of the kernel's own logits,
and the oracle's own pick equal unless its two candidates are within tolerance.
A second test uses weights whose picks are known in advance (a dominant
direction through ln_f) to pin the repetition-penalty dynamics exactly.
"""
import os

import numpy as np
import pytest
import torch

import oracle
from mockbird_b200 import KvRing, LocalHead, MockbirdError, argmax_penalty

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
H, HID = 12, 768
TOL_LOGIT = 2e-2   # bf16 weights and GEMM inputs through one layer and the head GEMM
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _layer_gains(w, h, ffn):
    """LayerNorm gains at 1 (ln1, ln2, ln_f) in a one-layer decoder block."""
    per = 2 * h + h * 3 * h + 3 * h + h * h + h + 2 * h + h * ffn + ffn + ffn * h + h
    w[0:h] = 1.0
    b2 = 2 * h + 3 * h * h + 3 * h + h * h + h
    w[b2:b2 + h] = 1.0
    w[per:per + h] = 1.0
    return per


def local_weights(h, ffn, codes, channels, seed):
    rng = np.random.default_rng(seed)
    n = LocalHead.weight_count(h, ffn, codes, channels)
    w = (rng.standard_normal(n) * 0.02).astype(np.float32)
    per = _layer_gains(w, h, ffn)
    off = per + 2 * h
    w[off:off + h] = rng.standard_normal(h)                                  # wte_slot
    off += h
    w[off:off + 2 * h] = rng.standard_normal(2 * h) / np.sqrt(h)             # text columns
    off += 2 * h
    m = (channels - 1) * codes * h
    w[off:off + m] = rng.standard_normal(m)                                  # audio embeddings
    return w


def _ring(streams, channels, dtype="f32", max_batch=0):
    return KvRing(layers=1, heads=H, capacity=channels + 1, streams=streams, dtype=dtype, wrap=False,
                  max_position=channels + 1, max_batch=max_batch)


# ------------------------------------------------------------------ ARGMAX_PENALTY alone

def test_argmax_kat_kernels_test5():
    """kernels.test.mjs test 5: 1024 xorshift32 logits, empty seen set: the id of
    the maximum (ties to the lowest id)."""
    kat = np.load(os.path.join(GOLDEN, "kat_argmax_c1024.npz"))
    rnd = oracle.xorshift32_stream(0x2F6E2B1)
    rnd(int(kat["skip"]), keep=False)
    logits = rnd(1024)
    assert abs(logits.astype(np.float64).sum() - float(kat["logits_sum"])) < 1e-9
    lg = torch.from_numpy(logits).to(DEV).reshape(1, -1)
    for penalty in (1.0, 1.2):
        seen = torch.zeros(1, 32, dtype=torch.int32, device=DEV)
        tok = argmax_penalty(lg, seen, penalty)
        assert int(tok[0]) == int(kat["best"])
        word = int(seen[0, int(kat["best"]) >> 5]) & 0xFFFFFFFF
        assert word == 1 << (int(kat["best"]) & 31)


def test_argmax_penalty_rules_and_random_rows():
    codes = 1024
    rows = []
    masks = []
    # ties: the lowest id wins
    r = np.zeros(codes, np.float32); r[[5, 700, 900]] = 3.0
    rows.append(r); masks.append(np.zeros(32, np.uint32))
    # a seen positive maximum is divided: 3.0/1.2 = 2.5 < 2.9
    r = np.zeros(codes, np.float32); r[10] = 3.0; r[20] = 2.9
    m = np.zeros(32, np.uint32); m[0] = 1 << 10
    rows.append(r); masks.append(m)
    # all negative: a seen maximum is multiplied: -1 * 1.2 = -1.2 < -1.1
    r = np.full(codes, -5.0, np.float32); r[40] = -1.0; r[41] = -1.1
    m = np.zeros(32, np.uint32); m[1] = 1 << (40 - 32)
    rows.append(r); masks.append(m)
    # nothing above -1e30: id 0 (the reference's starting point)
    rows.append(np.full(codes, -3e30, np.float32)); masks.append(np.zeros(32, np.uint32))
    # NaNs never win; a tie after the penalty: 2.4/1.2 == 2.0 exactly, the lower id wins
    r = np.zeros(codes, np.float32); r[3] = np.nan; r[600] = 2.0; r[50] = 2.4
    m = np.zeros(32, np.uint32); m[1] = 1 << (50 - 32)
    rows.append(r); masks.append(m)
    rng = np.random.default_rng(5)
    for _ in range(59):
        rows.append(rng.standard_normal(codes).astype(np.float32))
        masks.append(rng.integers(0, 2**32, size=32, dtype=np.uint64).astype(np.uint32)
                     & rng.integers(0, 2**32, size=32, dtype=np.uint64).astype(np.uint32))
    lg = np.stack(rows)
    seen = np.stack(masks)
    want = [oracle.argmax_penalty(lg[i], seen[i], 1.2) for i in range(len(rows))]
    assert want[:5] == [5, 20, 41, 0, 50]
    seen_dev = torch.from_numpy(seen.view(np.int32).copy()).to(DEV)
    got = argmax_penalty(torch.from_numpy(lg).to(DEV), seen_dev, 1.2).cpu().numpy()
    assert got.tolist() == want
    after = seen_dev.cpu().numpy().view(np.uint32)
    for i, t in enumerate(want):
        exp = seen[i].copy()
        exp[t >> 5] |= np.uint32(1 << (t & 31))
        assert np.array_equal(after[i], exp)


# ------------------------------------------------------------------ the whole head

@pytest.mark.parametrize("graph,heads,ffn,codes,channels", [
    ("1", H, 3072, 1024, 16),
    ("0", H, 3072, 1024, 16),
    ("1", 4, 512, 256, 4),   # a 256-wide layer: the other LayerNorm width of the fused embedding kernels
])
def test_local_frame_matches_oracle(graph, heads, ffn, codes, channels, monkeypatch):
    monkeypatch.setenv("MOCKBIRD_LOCAL_GRAPH", graph)
    h, penalty = heads * 64, 1.2
    S = 8
    order = [6, 1, 3, 0, 7]
    w = local_weights(h, ffn, codes, channels, seed=11)
    ring = KvRing(layers=1, heads=heads, capacity=channels + 1, streams=S, dtype="f32", wrap=False,
                  max_position=channels + 1)
    head = LocalHead(ring, w, ffn, codes, channels, penalty)
    orc = oracle.Ring(layers=1, streams=S, heads=heads, capacity=channels + 1, dtype="f32", wrap=False,
                      max_position=channels + 1)
    seen_o = np.zeros((S, channels, codes // 32), np.uint32)
    seen_k = np.zeros((S, channels, codes // 32), np.uint32)  # follows the kernel's picks
    rng = np.random.default_rng(2)
    worst, mismatches, checked = 0.0, 0, 0
    for frame in range(3):
        x = rng.standard_normal((len(order), h)).astype(np.float32)
        tok, cont, lg = head.frame(order, torch.from_numpy(x).to(DEV), logits=True)
        tok, cont, lg = tok.cpu().numpy(), cont.cpu().numpy(), lg.cpu().numpy()
        assert tok.min() >= 0 and tok.max() < codes
        for i, s in enumerate(order):
            for ch in range(channels):
                assert tok[i, ch] == oracle.argmax_penalty(lg[i, ch], seen_k[s, ch], penalty), (frame, i, ch)
                t = int(tok[i, ch])
                seen_k[s, ch, t >> 5] |= np.uint32(1 << (t & 31))
        before = seen_o.copy()
        tok_o, cont_o, lg_o, decide = oracle.local_frame(orc, w, ffn, codes, channels, penalty, order, x, seen_o,
                                                         forced=tok)
        worst = max(worst, float(np.abs(lg - lg_o).max()))
        for i, s in enumerate(order):
            for ch in range(channels):
                checked += 1
                if tok_o[i, ch] != tok[i, ch]:
                    mismatches += 1
                    pen = lg_o[i, ch].copy()
                    bits = ((before[s, ch][np.arange(codes) >> 5] >> (np.arange(codes) & 31)) & 1) != 0
                    pen[bits] = np.where(pen[bits] >= 0, pen[bits] / np.float32(penalty),
                                         pen[bits] * np.float32(penalty))
                    assert abs(float(pen[tok_o[i, ch]]) - float(pen[tok[i, ch]])) < 2 * TOL_LOGIT
            if cont_o[i] != cont[i]:
                assert abs(decide[i, 1] - decide[i, 0]) < TOL_LOGIT
        assert np.array_equal(seen_o, seen_k)
    ring.sync()
    assert worst < TOL_LOGIT, worst
    assert mismatches <= checked // 10, (mismatches, checked)
    head.dispose()


def _crafted_weights(h, ffn, codes, channels, seed=4):
    """ln_f gain 0.01 and bias u (signs): every step's ln_f output is ~u.  Audio
    heads 0..channels-2: column 3 = 10 u/h, column 7 = 9 u/h (others tiny), so a
    fresh channel picks 3, then 7 (10/1.2 < 9), then 3 (8.33 > 7.5).  The last
    head: column j = -10 (1 + 0.01 j) u/h (all logits negative), so frame f picks
    j = f while f < 20.  Text columns +-u/h: always continue."""
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal(LocalHead.weight_count(h, ffn, codes, channels)) * 0.02).astype(np.float32)
    per = _layer_gains(w, h, ffn)
    u = np.where(rng.standard_normal(h) >= 0, 1.0, -1.0).astype(np.float32)
    w[per:per + h] = 0.01
    w[per + h:per + 2 * h] = u
    off = per + 2 * h
    w[off:off + h] = rng.standard_normal(h)
    off += h
    w[off:off + h] = -u / h          # audio_end column
    w[off + h:off + 2 * h] = u / h   # assistant_slot column
    off += 2 * h
    m = (channels - 1) * codes * h
    w[off:off + m] = rng.standard_normal(m)
    off += m
    heads = (rng.standard_normal((channels, h, codes)) * 1e-4).astype(np.float32)
    heads[:channels - 1, :, 3] = 10.0 * u[None, :] / h
    heads[:channels - 1, :, 7] = 9.0 * u[None, :] / h
    heads[channels - 1] = (-10.0 * (1.0 + 0.01 * np.arange(codes))[None, :] * u[:, None] / h).astype(np.float32)
    w[off:] = heads.reshape(-1)
    return w


def test_local_penalty_dynamics_and_clear():
    h, ffn, codes, channels = HID, 1024, 1024, 16
    S = 4
    w = _crafted_weights(h, ffn, codes, channels)
    ring = _ring(S, channels, dtype="bf16")
    head = LocalHead(ring, w, ffn, codes, channels, 1.2)
    x = torch.randn(S, h, device=DEV)
    ids = list(range(S))
    pos_pattern = [3, 7, 3, 3]
    for frame in range(4):
        if frame == 2:
            head.clear(1)   # stream 1 starts a new utterance
        tok, cont, _ = head.frame(ids, x)
        tok, cont = tok.cpu().numpy(), cont.cpu().numpy()
        assert cont.tolist() == [1] * S
        for s in range(S):
            f = frame - 2 if (s == 1 and frame >= 2) else frame
            assert tok[s, :channels - 1].tolist() == [pos_pattern[f]] * (channels - 1), (frame, s)
            assert tok[s, channels - 1] == f, (frame, s)
    head.clear()            # all streams
    tok, _, _ = head.frame(ids, x)
    assert tok.cpu().numpy()[:, 0].tolist() == [3] * S
    ring.sync()
    head.dispose()


def test_local_head_rejects_bad_arguments():
    h, ffn, codes, channels = HID, 1024, 1024, 16
    w = local_weights(h, ffn, codes, channels, seed=0)
    with pytest.raises(MockbirdError):   # two layers
        LocalHead(KvRing(layers=2, capacity=17, streams=2, wrap=False), w, ffn, codes, channels)
    with pytest.raises(MockbirdError):   # 16 slots < 17 steps
        LocalHead(_ring(2, channels - 1), w, ffn, codes, channels)
    with pytest.raises(ValueError):
        LocalHead(_ring(2, channels), w[:-1], ffn, codes, channels)
    ring = _ring(2, channels)
    head = LocalHead(ring, w, ffn, codes, channels)
    with pytest.raises(MockbirdError):   # 3 items > max_batch 2
        head.frame([0, 1, 0], torch.zeros(3, h, device=DEV))
    with pytest.raises(MockbirdError):
        head.clear(2)
    head.dispose()


@pytest.mark.parametrize("graph", ["1", "0"])
def test_local_frame_host_arrays_match_device_arrays(graph, monkeypatch):
    """mb_local_head_frame_host (hidden rows from the host, tokens and stop flags
    back to the host, as nextFrame does) gives the device entry point's tokens and
    flags exactly, frame after frame (the seen masks carry over); bad stream ids
    are rejected on the host and the head stays usable."""
    monkeypatch.setenv("MOCKBIRD_LOCAL_GRAPH", graph)
    h, ffn, codes, channels, S = HID, 3072, 1024, 16, 6
    w = local_weights(h, ffn, codes, channels, seed=21)
    a = LocalHead(_ring(S, channels, dtype="bf16"), w, ffn, codes, channels, 1.2)
    b = LocalHead(_ring(S, channels, dtype="bf16"), w, ffn, codes, channels, 1.2)
    order = [4, 0, 5, 2]
    rng = np.random.default_rng(5)
    for frame in range(3):
        hidden = rng.standard_normal((len(order), h)).astype(np.float32)
        tok_a, cont_a, _ = a.frame(order, torch.from_numpy(hidden).to(DEV))
        tok_b, cont_b = b.frame_host(order, hidden)
        assert np.array_equal(tok_a.cpu().numpy(), tok_b), frame
        assert np.array_equal(cont_a.cpu().numpy(), cont_b), frame
    for bad in ([0, 0], [S], [-1]):
        with pytest.raises(MockbirdError) as e:
            b.frame_host(bad, np.zeros((len(bad), h), np.float32))
        assert e.value.status == "MB_ERR_STREAM"
    hidden = rng.standard_normal((2, h)).astype(np.float32)
    tok_a, cont_a, _ = a.frame([1, 3], torch.from_numpy(hidden).to(DEV))
    tok_b, cont_b = b.frame_host([1, 3], hidden)
    assert np.array_equal(tok_a.cpu().numpy(), tok_b) and np.array_equal(cont_a.cpu().numpy(), cont_b)
    a.dispose()
    b.dispose()


def test_local_frame_at_config6_batch():
    """The local head at the bench's batch: 256 streams in one frame (16 audio
    channels of 1024 codes, hidden 768, FFN 3072, graph replay), every logit row
    against the oracle and every pick against the penalised argmax of the
    kernel's own logits."""
    h, ffn, codes, channels, penalty, S = HID, 3072, 1024, 16, 1.2, 256
    w = local_weights(h, ffn, codes, channels, seed=12)
    ring = KvRing(layers=1, heads=H, capacity=channels + 1, streams=S, dtype="f32", wrap=False,
                  max_position=channels + 1)
    head = LocalHead(ring, w, ffn, codes, channels, penalty)
    orc = oracle.Ring(layers=1, streams=S, heads=H, capacity=channels + 1, dtype="f32", wrap=False,
                      max_position=channels + 1)
    order = list(np.random.default_rng(3).permutation(S))
    seen = np.zeros((S, channels, codes // 32), np.uint32)
    x = np.random.default_rng(4).standard_normal((S, h)).astype(np.float32)
    tok, cont, lg = head.frame(order, torch.from_numpy(x).to(DEV), logits=True)
    tok, lg = tok.cpu().numpy(), lg.cpu().numpy()
    for i in range(S):
        for ch in range(channels):
            assert tok[i, ch] == oracle.argmax_penalty(lg[i, ch], seen[order[i], ch], penalty), (i, ch)
    _, _, lg_o, _ = oracle.local_frame(orc, w, ffn, codes, channels, penalty, order, x, seen.copy(), forced=tok)
    ring.sync()
    assert float(np.abs(lg - lg_o).max()) < TOL_LOGIT
    head.dispose()
