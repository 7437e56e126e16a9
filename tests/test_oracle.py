"""CPU tests: the oracle against the reference's golden vectors, and its ring
semantics against small independent restatements.  No GPU needed."""
import os

import numpy as np
import pytest

import oracle

H, HD = 12, 64


def _golden(golden_dir, name):
    return np.load(os.path.join(golden_dir, name))


def _unrope_f64(k, pos, theta=10000.0):
    """Inverse rotation in fp64 (test-side restatement, independent of the oracle)."""
    inv = theta ** (-(2 * np.arange(32)) / 64.0)
    c, s = np.cos(pos * inv), np.sin(pos * inv)
    a = k[..., 0::2].astype(np.float64)
    b = k[..., 1::2].astype(np.float64)
    out = np.empty(k.shape, np.float64)
    out[..., 0::2] = a * c + b * s
    out[..., 1::2] = b * c - a * s
    return out


# ---------------------------------------------------------------- pins against the ONNX goldens

def test_fixture_is_consistent(golden_dir):
    g = _golden(golden_dir, "layer0_kv.npz")
    assert bool(g["k8_equal"]), "8-row goldens must be the prefix of the 195-row goldens"
    ids = g["ids"]
    assert ids.shape == (195, 17)
    # rows 131..194 of the Junhao prompt are the same row (64 identical frames)
    assert (ids[131:195] == ids[131]).all()
    assert (ids[2] == ids[4]).all()


def test_rope_convention_pinned_by_duplicate_rows(golden_dir):
    """Identical rows share pre-RoPE K at layer 0, so K[j] = RoPE_j(RoPE_i^-1(K[i]))."""
    g = _golden(golden_dir, "layer0_kv.npz")
    rows = list(g["rows"])
    K = {r: g["k"][i] for i, r in enumerate(rows)}
    tab = oracle.rope_table(256)
    pairs = [(2, 4)] + [(131, j) for j in range(132, 195)]
    worst = 0.0
    for i, j in pairs:
        raw = _unrope_f64(K[i], i).astype(np.float32).reshape(1, H * HD)
        got = oracle.rope_rows(raw, [j], tab).reshape(H, HD)
        worst = max(worst, float(np.abs(got - K[j]).max()))
    assert worst < 5e-5, worst  # ORT's own fp32 noise is ~1e-5
    # the opposite sign convention (kernels.test.mjs test 3's) is far off
    raw = _unrope_f64(K[131], 131)
    a, b = raw[..., 0::2], raw[..., 1::2]
    inv = 10000.0 ** (-(2 * np.arange(32)) / 64.0)
    c, s = np.cos(150 * inv), np.sin(150 * inv)
    flipped = np.empty_like(raw)
    flipped[..., 0::2] = a * c + b * s
    flipped[..., 1::2] = b * c - a * s
    assert np.abs(flipped - K[150]).max() > 0.1


def test_values_equal_for_duplicate_rows(golden_dir):
    g = _golden(golden_dir, "layer0_kv.npz")
    rows = list(g["rows"])
    V = {r: g["v"][i] for i, r in enumerate(rows)}
    for j in range(132, 195):
        assert np.array_equal(V[j], V[131])


def test_golden_kv_roundtrip_through_oracle_ring(golden_dir):
    """Golden layer-0 K/V as ring contents: written, wrapped and gathered bit-exactly."""
    g = _golden(golden_dir, "layer0_kv.npz")
    k = g["k"].astype(np.float32)  # [75][12][64]
    v = g["v"].astype(np.float32)
    ring = oracle.Ring(layers=1, streams=1, heads=H, capacity=32, dtype="f32", wrap=True)
    kv = ring.kv_view()
    for p in range(75):  # wraps twice
        kv[0, 0, 0, :, p % 32] = k[p]
        kv[0, 0, 1, :, p % 32] = v[p]
        ring.slot_pos[0, 0, p % 32] = p
    kk, vv, slots = ring.gather(0, 0, 74)
    assert list(slots) == [p % 32 for p in range(43, 75)]
    assert np.array_equal(kk, k[43:75].transpose(1, 0, 2))
    assert np.array_equal(vv, v[43:75].transpose(1, 0, 2))


# ---------------------------------------------------------------- known-answer test 4

def _kat_inputs():
    rnd = oracle.xorshift32_stream(0x2F6E2B1)
    kat = np.load(os.path.join(os.path.dirname(__file__), "golden", "kat_attention_n512.npz"))
    rnd(int(kat["skip"]), keep=False)
    kv = rnd(2 * 512 * H * HD)
    return kv[0::2].copy(), kv[1::2].copy(), rnd(H * HD), kat


def test_kat_attention_n512_oracle():
    """kernels.test.mjs test 4: attention of one query vs a 512-slot ring, 12 heads, tol 1e-5."""
    k, v, q, kat = _kat_inputs()
    assert abs(k.astype(np.float64).sum() - float(kat["k_sum"])) < 1e-6
    assert abs(v.astype(np.float64).sum() - float(kat["v_sum"])) < 1e-6
    assert abs(q.astype(np.float64).sum() - float(kat["q_sum"])) < 1e-9
    ring = oracle.Ring(layers=1, streams=1, heads=H, capacity=512, dtype="f32", wrap=False)
    kv = ring.kv_view()
    kv[0, 0, 0] = k.reshape(512, H, HD).transpose(1, 0, 2)   # test layout [slot][head][dim]
    kv[0, 0, 1] = v.reshape(512, H, HD).transpose(1, 0, 2)
    ring.slot_pos[0, 0, :] = np.arange(512)
    for mode in (0, 1):
        out = ring.attend(0, [0], [511], q.reshape(1, -1), mode=mode)
        err = float(np.abs(out[0] - kat["out"]).max())
        assert err < 1e-5, (mode, err)


# ---------------------------------------------------------------- pins of the decoder step's LayerNorm and GEMV

def test_kat_layernorm_d768_oracle():
    """kernels.test.mjs test 1: LayerNorm of one 768-row (x = 4 rnd(), g = 1,
    b = 0.1 rnd(), eps 1e-5), the test's own tolerance 2e-5.  This is the
    LayerNorm that `oracle.decoder_step` and `oracle.local_frame` apply, against
    which the CUDA decoder and local head are checked."""
    kat = np.load(os.path.join(os.path.dirname(__file__), "golden", "kat_layernorm_d768.npz"))
    d = oracle.xorshift32_stream_f64(0x2F6E2B1)(2 * H * HD)
    x = (d[0::2] * 4).astype(np.float32)
    b = (d[1::2] * 0.1).astype(np.float32)
    assert abs(x.astype(np.float64).sum() - float(kat["x_sum"])) < 1e-9
    assert abs(b.astype(np.float64).sum() - float(kat["b_sum"])) < 1e-12
    out = oracle.layer_norm(x[None, :], np.ones(H * HD, np.float32), b[None, :])[0]
    assert float(np.abs(out - kat["out"]).max()) < 2e-5


def test_kat_gemv_c_attn_oracle():
    """kernels.test.mjs test 2: y = bias + x W for the c_attn shape (K 768, N 2304),
    W = 0.05 rnd(), bias = 0.02 rnd(), the test's own tolerance 5e-3.  Checked at
    the CUDA path's rounding points (x and W rounded to bf16, exact products and
    sums), which is how `oracle.decoder_step` computes every GEMM of the layer,
    and in fp32 (no rounding of x or W), which must agree far closer."""
    kat = np.load(os.path.join(os.path.dirname(__file__), "golden", "kat_gemv_k768_n2304.npz"))
    K, N = H * HD, 3 * H * HD
    rnd = oracle.xorshift32_stream_f64(0x2F6E2B1)
    rnd(int(kat["skip"]))
    x = rnd(K).astype(np.float32)
    W = (rnd(K * N) * 0.05).astype(np.float32).reshape(K, N)
    bias = (rnd(N) * 0.02).astype(np.float32)
    assert abs(x.astype(np.float64).sum() - float(kat["x_sum"])) < 1e-9
    assert abs(W.astype(np.float64).sum() - float(kat["w_sum"])) < 1e-6
    assert abs(bias.astype(np.float64).sum() - float(kat["bias_sum"])) < 1e-12
    y = oracle.gemm_bf16(x[None, :], oracle.round_to("bf16", W), bias)[0]
    assert float(np.abs(y - kat["out"]).max()) < 5e-3
    y32 = (x.astype(np.float64) @ W.astype(np.float64) + bias).astype(np.float32)
    assert float(np.abs(y32 - kat["out"]).max()) < 1e-5


def test_fp64_draws_round_to_the_fp32_stream():
    """The fp64 draws, stored to fp32, are the fp32 stream's draws."""
    a = oracle.xorshift32_stream_f64(0x2F6E2B1)(4096)
    b = oracle.xorshift32_stream(0x2F6E2B1)(4096)
    assert np.array_equal(a.astype(np.float32), b)


# ---------------------------------------------------------------- ring semantics

def _np_attend(q, ks, vs):
    s = (ks.astype(np.float64) @ q.astype(np.float64)) * 0.125
    e = np.exp(s - s.max())
    return (e / e.sum()) @ vs.astype(np.float64)


@pytest.mark.parametrize("dtype", ["f32", "bf16", "f16"])
def test_ring_wrap_gather_and_attend(dtype):
    rng = np.random.default_rng(1)
    C, L, S = 8, 2, 3
    ring = oracle.Ring(layers=L, streams=S, heads=H, capacity=C, dtype=dtype, wrap=True)
    hist = {s: [] for s in range(S)}  # roped K (rounded) and V per stream per position, layer 1
    for pos in range(20):
        streams = [2, 0, 1]
        qkv = rng.standard_normal((3, 3 * H * HD)).astype(np.float32)
        ctx, roped = ring.append_attend(1, streams, [pos] * 3, qkv)
        for i, s in enumerate(streams):
            kr = oracle.rope_rows(qkv[i, H * HD:2 * H * HD].reshape(1, -1), [pos], ring.tab).reshape(H, HD)
            hist[s].append((oracle.round_to(dtype, kr), oracle.round_to(dtype, qkv[i, 2 * H * HD:].reshape(H, HD))))
            lo = max(0, pos - C + 1)
            ks = np.stack([hist[s][p][0] for p in range(lo, pos + 1)], 1)  # [H][W][64]
            vs = np.stack([hist[s][p][1] for p in range(lo, pos + 1)], 1)
            qr = roped[i, :H * HD].reshape(H, HD)
            ref = np.stack([_np_attend(qr[h], ks[h], vs[h]) for h in range(H)])
            tol = 2e-5 if dtype == "f32" else 1e-4
            assert np.abs(ctx[i].reshape(H, HD) - ref).max() < tol
    # slot j holds the latest position p <= 19 with p % C == j
    for s in range(S):
        assert list(ring.slot_pos[1, s]) == [max(p for p in range(20) if p % C == j) for j in range(C)]
        assert (ring.slot_pos[0, s] == -1).all()  # layer 0 untouched
        k, v, slots = ring.gather(1, s, 19)
        assert list(slots) == [p % C for p in range(12, 20)]
        if dtype == "f32":
            assert np.array_equal(k, np.stack([hist[s][p][0] for p in range(12, 20)], 1))
    ring.reset(1)
    assert (ring.slot_pos[:, 1] == -1).all() and (ring.slot_pos[1, 0] >= 0).all()


def test_holes_and_stale_slots_are_masked():
    """A skipped position leaves a slot holding an older position: it must not be attended."""
    rng = np.random.default_rng(2)
    C = 4
    ring = oracle.Ring(layers=1, streams=1, heads=H, capacity=C, dtype="f32", wrap=True)
    qkvs = {}
    for pos in [0, 1, 2, 3, 4, 6]:  # 5 skipped: slot 1 still holds position 1 (< 6 - 3)
        qkv = rng.standard_normal((1, 3 * H * HD)).astype(np.float32)
        qkvs[pos] = qkv
        ctx, roped = ring.append_attend(0, [0], [pos], qkv)
    k, v, slots = ring.gather(0, 0, 6)
    assert list(slots) == [3, 0, -1, 2]   # positions 3, 4, (5 missing), 6
    assert (k[:, 2] == 0).all()
    # attention over positions {3, 4, 6} only
    kr = {p: oracle.rope_rows(qkvs[p][:, H * HD:2 * H * HD], [p], ring.tab).reshape(H, HD) for p in (3, 4, 6)}
    vr = {p: qkvs[p][0, 2 * H * HD:].reshape(H, HD) for p in (3, 4, 6)}
    qr = roped[0, :H * HD].reshape(H, HD)
    for h in range(H):
        ref = _np_attend(qr[h], np.stack([kr[p][h] for p in (3, 4, 6)]), np.stack([vr[p][h] for p in (3, 4, 6)]))
        assert np.abs(ctx[0].reshape(H, HD)[h] - ref).max() < 2e-5


def test_non_wrapping_ring_rejects_overflow():
    ring = oracle.Ring(layers=1, streams=1, heads=H, capacity=4, dtype="f32", wrap=False)
    qkv = np.zeros((1, 3 * H * HD), np.float32)
    for pos in range(4):
        ring.rope_split(0, [0], [pos], qkv)
    with pytest.raises(ValueError):
        ring.rope_split(0, [0], [4], qkv)


def test_prefill_oracle_matches_fp64_causal_attention():
    rng = np.random.default_rng(3)
    rows = 37
    ring = oracle.Ring(layers=1, streams=2, heads=H, capacity=64, dtype="f32", wrap=False)
    qkv = (rng.standard_normal((1, rows, 3 * H * HD)) * 0.5).astype(np.float32)
    ctx, roped = ring.prefill(0, [1], qkv)
    q = roped[0, :, :H * HD].reshape(rows, H, HD)
    k = oracle.rope_rows(qkv[0, :, H * HD:2 * H * HD], np.arange(rows), ring.tab).reshape(rows, H, HD)
    v = qkv[0, :, 2 * H * HD:].reshape(rows, H, HD)
    for h in range(H):
        for t in range(rows):
            ref = _np_attend(q[t, h], k[:t + 1, h], v[:t + 1, h])
            assert np.abs(ctx[0, t].reshape(H, HD)[h] - ref).max() < 2e-5
    assert list(ring.slot_pos[0, 1, :rows]) == list(range(rows))
    assert (ring.slot_pos[0, 0] == -1).all()
    kk, _, _ = ring.gather(0, 1, rows - 1)
    assert np.array_equal(kk, k.transpose(1, 0, 2))


def test_storage_rounding_matches_numpy():
    x = np.random.default_rng(4).standard_normal(4096).astype(np.float32) * 37.0
    assert np.array_equal(oracle.round_to("f16", x), x.astype(np.float16).astype(np.float32))
    u = x.view(np.uint32).astype(np.uint64)
    bf = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint32) << 16
    assert np.array_equal(oracle.round_to("bf16", x), bf.astype(np.uint32).view(np.float32))


# ---------------------------------------------------------------- local head (ARGMAX_PENALTY, nextFrame)

def test_kat_argmax_c1024_oracle():
    """kernels.test.mjs test 5: the id of the maximum of 1024 xorshift32 logits."""
    kat = np.load(os.path.join(os.path.dirname(__file__), "golden", "kat_argmax_c1024.npz"))
    rnd = oracle.xorshift32_stream(0x2F6E2B1)
    rnd(int(kat["skip"]), keep=False)
    logits = rnd(1024)
    assert abs(logits.astype(np.float64).sum() - float(kat["logits_sum"])) < 1e-9
    assert oracle.argmax_penalty(logits, np.zeros(32, np.uint32), 1.0) == int(kat["best"])
    # with its own bit set, the maximum is divided by 1.2 and the runner-up may win
    seen = np.zeros(32, np.uint32)
    seen[int(kat["best"]) >> 5] = np.uint32(1 << (int(kat["best"]) & 31))
    pen = logits.copy()
    pen[int(kat["best"])] = pen[int(kat["best"])] / np.float32(1.2)
    assert oracle.argmax_penalty(logits, seen, 1.2) == int(np.argmax(pen))


def test_oracle_local_frame_penalty_dynamics():
    """A small local head whose picks are known in advance: ln_f gain 0.01 and bias
    u make every step's output ~u; heads 0..1 favour id 3 (10 u/h) over id 7
    (9 u/h), so a channel picks 3, 7 (10/1.2 < 9), 3, 3; head 2 has all-negative
    logits -10 (1 + 0.01 j), so frame f picks j = f.  Stream 1 is cleared before
    frame 2 and starts over."""
    h, ffn, codes, channels = 64, 64, 64, 3
    rng = np.random.default_rng(0)
    n = oracle.local_weight_count(h, ffn, codes, channels)
    w = (rng.standard_normal(n) * 0.02).astype(np.float32)
    per = 2 * h + h * 3 * h + 3 * h + h * h + h + 2 * h + h * ffn + ffn + ffn * h + h
    w[0:h] = 1.0
    w[2 * h + 3 * h * h + 3 * h + h * h + h: 2 * h + 3 * h * h + 3 * h + h * h + 2 * h] = 1.0
    u = np.where(rng.standard_normal(h) >= 0, 1.0, -1.0).astype(np.float32)
    w[per:per + h] = 0.01
    w[per + h:per + 2 * h] = u
    off = per + 2 * h + h
    w[off:off + h] = -u / h
    w[off + h:off + 2 * h] = u / h
    off += 2 * h + (channels - 1) * codes * h
    heads = (rng.standard_normal((channels, h, codes)) * 1e-4).astype(np.float32)
    heads[:channels - 1, :, 3] = 10.0 * u / h
    heads[:channels - 1, :, 7] = 9.0 * u / h
    heads[channels - 1] = -10.0 * (1.0 + 0.01 * np.arange(codes))[None, :] * u[:, None] / h
    w[off:] = heads.reshape(-1)
    S = 2
    ring = oracle.Ring(layers=1, streams=S, heads=1, capacity=channels + 1, dtype="f32", wrap=False,
                       max_position=channels + 1)
    seen = np.zeros((S, channels, codes // 32), np.uint32)
    x = rng.standard_normal((S, h)).astype(np.float32)
    pattern = [3, 7, 3, 3]
    for frame in range(4):
        if frame == 2:
            seen[1] = 0
        tok, cont, _, _ = oracle.local_frame(ring, w, ffn, codes, channels, 1.2, [0, 1], x, seen)
        assert cont.tolist() == [1, 1]
        for s in range(S):
            f = frame - 2 if (s == 1 and frame >= 2) else frame
            assert tok[s].tolist() == [pattern[f]] * (channels - 1) + [f], (frame, s)
