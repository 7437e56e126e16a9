"""GPU parity of the decode path (append + RoPE + flash-decode), through the C ABI,
against the CPU oracle.  Ring bytes, slot indices and wrap order bit-exact;
attention within max-abs 2e-3 (fp32 storage) / 1e-2 (fp16, bf16 storage)."""
import os

import numpy as np
import pytest
import torch

import oracle
from gpu_util import HD, HID, QKV, TOL, H, assert_window_equal, from_np_storage, max_err, randn, to_np_storage  # noqa: F401
from mockbird_b200 import KvRing, MockbirdError

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


@pytest.mark.parametrize("dtype", ["f32", "bf16", "f16"])
def test_wrapping_ring_parity(dtype):
    """Streams appended out of order, two of them starting late, the ring wrapping
    more than twice, several split-K chunks per window."""
    L, S, C = 2, 6, 200
    ring = KvRing(layers=L, streams=S, capacity=C, dtype=dtype, wrap=True)
    orc = oracle.Ring(layers=L, streams=S, heads=H, capacity=C, dtype=dtype, wrap=True)
    start = {5: 0, 0: 0, 3: 0, 2: 0, 1: 100, 4: 137}
    worst = 0.0
    for step in range(460):
        items = [s for s in (5, 0, 3, 2, 1, 4) if step >= start[s]]
        pos = [step - start[s] for s in items]
        for layer in range(L):
            qkv = randn((len(items), QKV), seed=step * 10 + layer)
            out = ring.append_attend(layer, items, pos, torch.from_numpy(qkv).to(DEV))
            ref, _ = orc.append_attend(layer, items, pos, qkv)
            worst = max(worst, max_err(out, ref))
        if step % 97 == 0 or step == 459:
            ring.sync()
            for layer in range(L):
                for s, p in zip(items, pos):
                    assert_window_equal(ring, orc, layer, s, layer, s, p)
    ring.sync()
    assert worst < TOL[dtype], worst


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_fused_equals_rope_then_attend(dtype):
    """mb_append_attend == mb_rope_append + mb_attend, bit for bit; roped Q bit-exact."""
    S, C = 4, 300
    a = KvRing(layers=1, streams=S, capacity=C, dtype=dtype, wrap=True)
    b = KvRing(layers=1, streams=S, capacity=C, dtype=dtype, wrap=True)
    tab = oracle.rope_table(1024)
    for step in range(350):
        qkv = torch.from_numpy(randn((S, QKV), seed=step)).to(DEV)
        pos = [step] * S
        oa = a.append_attend(0, [0, 1, 2, 3], pos, qkv)
        qb = qkv.clone()
        b.rope_split_ring(0, [0, 1, 2, 3], pos, qb)
        ob = b.attend_ring(0, [0, 1, 2, 3], pos, qb, q_stride=QKV)
        assert torch.equal(oa, ob), step
        if step in (0, 63, 64, 299, 300, 349):
            ref_q = oracle.rope_rows(qkv[:, :HID].cpu().numpy(), pos, tab)
            assert np.array_equal(qb[:, :HID].cpu().numpy(), ref_q)
            assert torch.equal(qb[:, HID:], qkv[:, HID:])  # K/V part of the row untouched
    a.sync()
    b.sync()


def test_kat_attention_n512_gpu():
    """kernels.test.mjs test 4 (N=512, 12 heads) within its own tolerance 1e-5."""
    kat = np.load(os.path.join(GOLDEN, "kat_attention_n512.npz"))
    rnd = oracle.xorshift32_stream(0x2F6E2B1)
    rnd(int(kat["skip"]), keep=False)
    kv = rnd(2 * 512 * H * HD)
    k = kv[0::2].reshape(512, H, HD).transpose(1, 0, 2).copy()
    v = kv[1::2].reshape(512, H, HD).transpose(1, 0, 2).copy()
    q = rnd(H * HD)
    ring = KvRing(layers=1, streams=1, capacity=512, dtype="f32", wrap=False)
    ring.ring_write(0, 0, 0, torch.from_numpy(k).to(DEV), torch.from_numpy(v).to(DEV))
    out = ring.attend_ring(0, [0], [511], torch.from_numpy(q.reshape(1, -1)).to(DEV))
    ring.sync()
    assert max_err(out[0], kat["out"]) < 1e-5


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_golden_kv_as_ring_contents(dtype):
    """The ONNX layer-0 K/V rows as realistic ring contents, wrapped, vs the fp64 oracle."""
    g = np.load(os.path.join(GOLDEN, "layer0_kv.npz"))
    k = np.ascontiguousarray(g["k"].transpose(1, 0, 2))  # [12][75][64]
    v = np.ascontiguousarray(g["v"].transpose(1, 0, 2))
    C = 48
    ring = KvRing(layers=1, streams=1, capacity=C, dtype=dtype, wrap=True)
    orc = oracle.Ring(layers=1, streams=1, heads=H, capacity=C, dtype=dtype, wrap=True)
    ks = oracle.round_to(dtype, k)
    vs = oracle.round_to(dtype, v)
    ring.ring_write(0, 0, 27, from_np_storage(_to_storage(ks[:, 27:], dtype), dtype),
                    from_np_storage(_to_storage(vs[:, 27:], dtype), dtype))
    kvv = orc.kv_view()
    for p in range(27, 75):
        kvv[0, 0, 0, :, p % C] = _to_storage(ks[:, p], dtype)
        kvv[0, 0, 1, :, p % C] = _to_storage(vs[:, p], dtype)
        orc.slot_pos[0, 0, p % C] = p
    q = randn((1, HID), seed=7)
    out = ring.attend_ring(0, [0], [74], torch.from_numpy(q).to(DEV))
    ref = orc.attend(0, [0], [74], q, mode=1)
    ring.sync()
    assert_window_equal(ring, orc, 0, 0, 0, 0, 74)
    assert max_err(out, ref) < TOL[dtype]


def _to_storage(x, dtype):
    if dtype == "f32":
        return np.ascontiguousarray(x, np.float32)
    if dtype == "f16":
        return np.ascontiguousarray(x, np.float32).astype(np.float16).view(np.uint16)
    u = np.ascontiguousarray(x, np.float32).view(np.uint32)
    return (u >> 16).astype(np.uint16)  # x is already bf16-representable


def test_config1_single_stream_step():
    """1 stream, 12 layers, C=2048, slots 0..299 filled with
    N(0,1) K/V (seed 0), append + attend at position 300 (RoPE theta 10000)."""
    ring = KvRing(layers=12, streams=1, capacity=2048, dtype="f32", wrap=False)
    orc = oracle.Ring(layers=12, streams=1, heads=H, capacity=2048, dtype="f32", wrap=False)
    rng = np.random.default_rng(0)
    for layer in range(12):
        k = rng.standard_normal((H, 300, HD)).astype(np.float32)
        v = rng.standard_normal((H, 300, HD)).astype(np.float32)
        ring.ring_write(layer, 0, 0, torch.from_numpy(k).to(DEV), torch.from_numpy(v).to(DEV))
        orc.kv_view()[layer, 0, 0, :, :300] = k
        orc.kv_view()[layer, 0, 1, :, :300] = v
        orc.slot_pos[layer, 0, :300] = np.arange(300)
    qkv = np.random.default_rng(0).standard_normal((12, 1, QKV)).astype(np.float32)
    for layer in range(12):
        out = ring.append_attend(layer, [0], [300], torch.from_numpy(qkv[layer]).to(DEV))
        ref, _ = orc.append_attend(layer, [0], [300], qkv[layer])
        ref64 = orc.attend(layer, [0], [300], _, mode=1)
        assert max_err(out, ref) < TOL["f32"]
        assert max_err(out, ref64) < TOL["f32"]
        assert_window_equal(ring, orc, layer, 0, layer, 0, 300)
    ring.sync()


def test_config2_full_size_wrap_properties():
    """BASELINE config 2 at full size: 64 streams x 12 layers, fp32, C=512, 1500
    appends (two wraps).  The GPU runs everything; the oracle replays 2 layers x 3
    streams in lockstep; the final ring order is checked for all streams."""
    L, S, C, STEPS = 12, 64, 512, 1500
    ring = KvRing(layers=L, streams=S, capacity=C, dtype="f32", wrap=True)
    track = [(0, 0), (7, 33), (11, 63)]  # (layer, stream)
    orc = oracle.Ring(layers=len(track), streams=1, heads=H, capacity=C, dtype="f32", wrap=True)
    streams = torch.arange(S, dtype=torch.int32, device=DEV)
    gen = torch.Generator(device=DEV)
    worst = 0.0
    check_steps = {0, 1, 511, 512, 513, 1023, 1024, 1499}
    for step in range(STEPS):
        gen.manual_seed(step)
        qkv = torch.randn(L, S, QKV, generator=gen, device=DEV)
        pos = torch.full((S,), step, dtype=torch.int32, device=DEV)
        outs = [ring.append_attend(layer, streams, pos, qkv[layer]) for layer in range(L)]
        sub = [qkv[layer, s].cpu().numpy()[None] for layer, s in track]
        for t, (layer, s) in enumerate(track):
            ref, _ = orc.append_attend(t, [0], [step], sub[t])
            if step in check_steps:
                worst = max(worst, max_err(outs[layer][s], ref[0]))
    ring.sync()
    assert worst < TOL["f32"], worst
    for t, (layer, s) in enumerate(track):
        assert_window_equal(ring, orc, layer, s, t, 0, STEPS - 1)
    expected = np.array([p % C for p in range(STEPS - C, STEPS)], np.int32)
    for s in range(S):
        _, _, slots = ring.gather(5, s, STEPS - 1)
        assert np.array_equal(slots.cpu().numpy(), expected)


def test_variable_live_lengths_bf16():
    """Config-5 style: per-stream live lengths U[1, C] (seeded), bf16, 24 steps of
    appends (some streams wrap), all streams in one launch."""
    S, C = 16, 512
    rng = np.random.default_rng(5)
    lengths = rng.integers(1, C + 1, size=S)
    ring = KvRing(layers=1, streams=S, capacity=C, dtype="bf16", wrap=True)
    orc = oracle.Ring(layers=1, streams=S, heads=H, capacity=C, dtype="bf16", wrap=True)
    for s in range(S):
        n = int(lengths[s]) - 1
        if n == 0:
            continue
        k = _to_storage(oracle.round_to("bf16", rng.standard_normal((H, n, HD)).astype(np.float32)), "bf16")
        v = _to_storage(oracle.round_to("bf16", rng.standard_normal((H, n, HD)).astype(np.float32)), "bf16")
        ring.ring_write(0, s, 0, from_np_storage(k, "bf16"), from_np_storage(v, "bf16"))
        orc.kv_view()[0, s, 0, :, :n] = k
        orc.kv_view()[0, s, 1, :, :n] = v
        orc.slot_pos[0, s, :n] = np.arange(n)
    order = list(rng.permutation(S))
    worst = 0.0
    for step in range(24):
        pos = [int(lengths[s]) - 1 + step for s in order]
        qkv = randn((S, QKV), seed=1000 + step)
        out = ring.append_attend(0, order, pos, torch.from_numpy(qkv).to(DEV))
        ref, _ = orc.append_attend(0, order, pos, qkv)
        worst = max(worst, max_err(out, ref))
    ring.sync()
    assert worst < TOL["bf16"], worst
    for s, p in zip(order, pos):
        assert_window_equal(ring, orc, 0, s, 0, s, p)


def test_config5_shape_long_uneven_windows_bf16():
    """BASELINE config 5's shape: bf16 ring of C = 4096 slots, 64 streams with
    seeded live lengths U[1, 4096], 200 consecutive steps of appends, all streams
    in one launch per step.  Windows reach 32 split-K chunks (the path without the
    L2 prefetch, taken above 16 chunks), and the longest streams wrap during the
    run.  The oracle replays 8 of the streams in lockstep (the 3 longest, the 2
    shortest, 3 others): contexts within 1e-2 of its fp32 mirror and of its fp64
    mode; their windows bit-exact; the final slot order of all 64 streams."""
    S, C, STEPS = 64, 4096, 200
    rng = np.random.default_rng(2024)
    lengths = rng.integers(1, C + 1, size=S)
    by_len = np.argsort(lengths)
    others = [s for s in rng.permutation(S) if s not in set(by_len[:2]) | set(by_len[-3:])][:3]
    track = [int(x) for x in list(by_len[-3:]) + list(by_len[:2]) + others]
    assert lengths[track[0]] + STEPS - 1 > C, "the longest tracked stream must wrap"
    ring = KvRing(layers=1, streams=S, capacity=C, dtype="bf16", wrap=True, max_position=8192)
    orc = oracle.Ring(layers=1, streams=len(track), heads=H, capacity=C, dtype="bf16", wrap=True,
                      max_position=8192)
    gen = torch.Generator(device=DEV)
    gen.manual_seed(11)
    for s in range(S):  # positions 0..L-2 of every stream, N(0, 1) rows rounded to bf16
        n = int(lengths[s]) - 1
        if n == 0:
            continue
        k = torch.randn(H, n, HD, generator=gen, device=DEV).to(torch.bfloat16)
        v = torch.randn(H, n, HD, generator=gen, device=DEV).to(torch.bfloat16)
        ring.ring_write(0, s, 0, k, v)
        if s in track:
            t = track.index(s)
            orc.kv_view()[0, t, 0, :, :n] = to_np_storage(k)
            orc.kv_view()[0, t, 1, :, :n] = to_np_storage(v)
            orc.slot_pos[0, t, :n] = np.arange(n)
    order = [int(x) for x in rng.permutation(S)]
    rows = [order.index(s) for s in track]
    worst = worst64 = 0.0
    for step in range(STEPS):
        pos = [int(lengths[s]) - 1 + step for s in order]
        qkv = randn((S, QKV), seed=7000 + step)
        out = ring.append_attend(0, order, pos, torch.from_numpy(qkv).to(DEV)).cpu().numpy()
        tpos = [pos[r] for r in rows]
        ref, q_roped = orc.append_attend(0, list(range(len(track))), tpos, qkv[rows])
        worst = max(worst, max_err(out[rows], ref))
        if step % 25 == 0 or step == STEPS - 1:
            ref64 = orc.attend(0, list(range(len(track))), tpos, q_roped, mode=1)
            worst64 = max(worst64, max_err(out[rows], ref64))
        if step in (0, 99):
            ring.sync()
            for t, s in enumerate(track):
                assert_window_equal(ring, orc, 0, s, 0, t, tpos[t])
    ring.sync()
    assert worst < TOL["bf16"], worst
    assert worst64 < TOL["bf16"], worst64
    for t, s in enumerate(track):
        assert_window_equal(ring, orc, 0, s, 0, t, int(lengths[s]) - 1 + STEPS - 1)
    for s in range(S):
        p = int(lengths[s]) - 1 + STEPS - 1
        W = min(p + 1, C)
        _, _, slots = ring.gather(0, s, p)
        assert np.array_equal(slots.cpu().numpy(), np.array([q % C for q in range(p - W + 1, p + 1)], np.int32)), s


def test_host_entry_points_match_device_path():
    S, C, L = 3, 128, 12
    a = KvRing(layers=L, streams=S, capacity=C, dtype="f32", wrap=True)
    b = KvRing(layers=L, streams=S, capacity=C, dtype="f32", wrap=True)
    c = KvRing(layers=L, streams=S, capacity=C, dtype="f32", wrap=True)
    for step in range(140):
        qkv = randn((L, S, QKV), seed=step)
        pos = [step, step, step]
        host = a.decode_step_host([2, 0, 1], pos, qkv)
        for layer in range(L):
            dev = b.append_attend(layer, [2, 0, 1], pos, torch.from_numpy(qkv[layer]).to(DEV))
            one = c.append_attend_host(layer, [2, 0, 1], pos, qkv[layer])
            assert np.array_equal(host[layer], dev.cpu().numpy())
            assert np.array_equal(one, host[layer])


def test_host_step_with_shared_copy_groups_matches_device_path():
    """Windows long enough (64 streams x 512 fp32 slots) that the host step runs
    several layers per launch and copies their rows in and out as one group;
    results equal the device path bit for bit, layer by layer."""
    S, C, L = 64, 512, 12
    a = KvRing(layers=L, streams=S, capacity=C, dtype="f32", wrap=True)
    b = KvRing(layers=L, streams=S, capacity=C, dtype="f32", wrap=True)
    order = list(np.random.default_rng(3).permutation(S))
    for step in range(4):
        qkv = randn((L, S, QKV), seed=500 + step)
        pos = [700 + step + (s % 5) for s in order]
        host = a.decode_step_host(order, pos, qkv)
        for layer in range(L):
            dev = b.append_attend(layer, order, pos, torch.from_numpy(qkv[layer]).to(DEV))
            assert np.array_equal(host[layer], dev.cpu().numpy()), (step, layer)


def test_empty_batches_are_no_ops():
    """A call with no items succeeds on every decode and prefill entry point and
    leaves the ring as it was (bytes and slot positions)."""
    ring = KvRing(layers=2, streams=3, capacity=64, dtype="f32", wrap=True)
    orc = oracle.Ring(layers=2, streams=3, heads=H, capacity=64, dtype="f32", wrap=True)
    for p in range(5):
        qkv = randn((3, QKV), seed=40 + p)
        ring.append_attend(1, [0, 1, 2], [p] * 3, torch.from_numpy(qkv).to(DEV))
        orc.append_attend(1, [0, 1, 2], [p] * 3, qkv)
    none = torch.empty(0, dtype=torch.int32, device=DEV)
    q0 = torch.empty(0, QKV, device=DEV)
    assert ring.append_attend(1, none, none, q0).shape == (0, HID)
    assert ring.rope_split_ring(1, none, none, q0).shape == (0, QKV)
    assert ring.attend_ring(1, none, none, q0).shape == (0, HID)
    assert ring.decode_step(none, none, torch.empty(2, 0, QKV, device=DEV)).shape == (2, 0, HID)
    assert ring.append_attend_host(1, [], [], np.empty((0, QKV), np.float32)).shape == (0, HID)
    assert ring.decode_step_host([], [], np.empty((2, 0, QKV), np.float32)).shape == (2, 0, HID)
    assert ring.prefill(0, none, torch.empty(0, 8, QKV, device=DEV)).shape == (0, 8, HID)
    ring.sync()
    for s in range(3):
        assert_window_equal(ring, orc, 1, s, 1, s, 4)


def test_errors_are_reported_and_the_context_survives():
    ring = KvRing(layers=2, streams=4, capacity=8, dtype="f32", wrap=False, max_batch=4)
    qkv = randn((1, QKV), seed=0)
    for p in range(8):
        ring.append_attend_host(0, [1], [p], qkv)
    with pytest.raises(MockbirdError, match="exceeds the KV ring") as e:
        ring.append_attend_host(0, [1], [8], qkv)
    assert e.value.status == "MB_ERR_CAPACITY"
    with pytest.raises(MockbirdError) as e:
        ring.append_attend_host(0, [4], [0], qkv)
    assert e.value.status == "MB_ERR_STREAM"
    with pytest.raises(MockbirdError) as e:
        ring.append_attend_host(0, [1, 1], [0, 0], np.concatenate([qkv, qkv]))
    assert e.value.status == "MB_ERR_STREAM"
    with pytest.raises(MockbirdError) as e:
        ring.append_attend_host(2, [1], [0], qkv)
    assert e.value.status == "MB_ERR_LAYER"
    with pytest.raises(MockbirdError) as e:
        ring.append_attend_host(0, [0], [-1], qkv)
    assert e.value.status == "MB_ERR_POSITION"
    with pytest.raises(MockbirdError) as e:
        ring.append_attend_host(0, [0, 1, 2, 3, 0], [0] * 5, np.repeat(qkv, 5, 0))
    assert e.value.status == "MB_ERR_ARG"
    # device-side rejection: the bad item is skipped, the good one is computed
    good = KvRing(layers=2, streams=4, capacity=8, dtype="f32", wrap=False)
    q2 = torch.from_numpy(randn((2, QKV), seed=3)).to(DEV)
    out = ring.append_attend(1, torch.tensor([0, 9], dtype=torch.int32, device=DEV),
                             torch.tensor([0, 0], dtype=torch.int32, device=DEV), q2)
    with pytest.raises(MockbirdError) as e:
        ring.sync()
    assert e.value.status == "MB_ERR_DEVICE"
    ref = good.append_attend(1, [0], [0], q2[:1].clone())
    assert torch.equal(out[0], ref[0])
    ring.append_attend(1, torch.tensor([2], dtype=torch.int32, device=DEV),
                       torch.tensor([8], dtype=torch.int32, device=DEV), q2[:1].clone())
    with pytest.raises(MockbirdError, match="non-wrapping"):
        ring.sync()
    ring.sync()  # status cleared
    # and the context still computes correctly
    orc = oracle.Ring(layers=2, streams=4, heads=H, capacity=8, dtype="f32", wrap=False)
    for p in range(8):
        orc.append_attend(0, [1], [p], qkv)
    q3 = randn((1, QKV), seed=9)
    ring.reset(1)
    orc.reset(1)
    out = ring.append_attend_host(0, [1], [0], q3)
    ref, _ = orc.append_attend(0, [1], [0], q3)
    assert max_err(out, ref) < TOL["f32"]


def test_empty_window_reset_and_poison_readback():
    ring = KvRing(layers=1, streams=2, capacity=16, dtype="f32", wrap=True)
    q = torch.from_numpy(randn((1, HID), seed=1)).to(DEV)
    out = ring.attend_ring(0, [1], [5], q)
    assert torch.count_nonzero(out).item() == 0  # nothing live: zeros, not NaN
    # the warm-up check of gpu.ts:201-234: poison, read back, then overwrite
    ring.poison_kv(0, 0, 2)
    k, v = ring.read_layer_cache(0, 0, 2)
    assert torch.all(k == -12345.5) and torch.all(v == -12345.5)
    qkv = torch.from_numpy(randn((2, QKV), seed=2)).to(DEV)
    ring.append_attend(0, [0], [0], qkv[:1].clone())
    ring.append_attend(0, [0], [1], qkv[1:].clone())
    k, v = ring.read_layer_cache(0, 0, 2)
    assert not torch.any(k == -12345.5)
    ring.reset()
    out = ring.attend_ring(0, [0], [1], q)
    assert torch.count_nonzero(out).item() == 0
    ring.sync()


@pytest.mark.parametrize("dtype,C,items", [("f32", 512, 64), ("bf16", 4096, 3), ("f16", 256, 37)])
def test_persistent_and_chunked_kernels_agree(dtype, C, items, monkeypatch):
    """The per-chunk decode kernel (default) and the persistent stream-K kernel
    (MOCKBIRD_DECODE_KERNEL=persistent) compute the same thing: identical ring bytes, contexts within fp32 rounding, and both
    within the oracle tolerance.  Windows of varied length, some split across CTAs."""
    rings = {}
    for kernel in ("persistent", "chunked"):
        monkeypatch.setenv("MOCKBIRD_DECODE_KERNEL", kernel)
        rings[kernel] = KvRing(layers=2, streams=items, capacity=C, dtype=dtype, wrap=True)
    orc = oracle.Ring(layers=2, streams=items, heads=H, capacity=C, dtype=dtype, wrap=True)
    rng = np.random.default_rng(11)
    start = rng.integers(0, 3 * C, size=items)  # streams at different points, some already wrapped
    for s in range(items):  # jump-start: write the positions before start[s] directly
        first = max(0, int(start[s]) - C)
        cnt = int(start[s]) - first
        if cnt == 0:
            continue
        k = oracle.round_to(dtype, rng.standard_normal((H, cnt, HD)).astype(np.float32))
        v = oracle.round_to(dtype, rng.standard_normal((H, cnt, HD)).astype(np.float32))
        for ring in rings.values():
            for layer in range(2):
                ring.ring_write(layer, s, first, from_np_storage(_to_storage(k, dtype), dtype),
                                from_np_storage(_to_storage(v, dtype), dtype))
        for layer in range(2):
            for w in range(cnt):
                p = first + w
                orc.kv_view()[layer, s, 0, :, p % C] = _to_storage(k[:, w], dtype)
                orc.kv_view()[layer, s, 1, :, p % C] = _to_storage(v[:, w], dtype)
                orc.slot_pos[layer, s, p % C] = p
    order = list(rng.permutation(items))
    worst = {"persistent": 0.0, "chunked": 0.0}
    for step in range(6):
        pos = [int(start[s]) + step for s in order]
        qkv = randn((items, QKV), seed=700 + step)
        outs = {kname: ring.append_attend(step % 2, order, pos, torch.from_numpy(qkv).to(DEV))
                for kname, ring in rings.items()}
        ref, _ = orc.append_attend(step % 2, order, pos, qkv)
        for kname, o in outs.items():
            worst[kname] = max(worst[kname], max_err(o, ref))
        assert max_err(outs["persistent"], outs["chunked"]) < 1e-5
    for ring in rings.values():
        ring.sync()
    for kname in rings:
        assert worst[kname] < TOL[dtype], (kname, worst)
    for s, p in zip(order, pos):
        ka, va, sa = rings["persistent"].gather(1, s, p)
        kb, vb, sb = rings["chunked"].gather(1, s, p)
        assert torch.equal(sa, sb) and torch.equal(ka, kb) and torch.equal(va, vb)
        assert_window_equal(rings["persistent"], orc, 1, s, 1, s, p)


def test_many_streams_take_the_chunked_kernel():
    """More items than the persistent kernel's prologue holds (2048): same results."""
    S, C = 2100, 8
    ring = KvRing(layers=1, streams=S, capacity=C, dtype="f32", wrap=True)
    orc = oracle.Ring(layers=1, streams=S, heads=H, capacity=C, dtype="f32", wrap=True)
    for step in range(10):
        qkv = randn((S, QKV), seed=900 + step)
        out = ring.append_attend(0, np.arange(S), [step] * S, torch.from_numpy(qkv).to(DEV))
        ref, _ = orc.append_attend(0, np.arange(S), [step] * S, qkv)
        assert max_err(out, ref) < TOL["f32"]
    ring.sync()


@pytest.mark.parametrize("capacity", [500, 1696, 2480, 3248])
def test_codec_ring_geometry(capacity):
    """The codec decoder's rings (codec.ts:1-28, 204-225): d = 256 = 4 heads x 64,
    wrapping capacities 500 / 1696 / 2480 / 3248, fp32, slot = pos % C with the
    stored-position mask (ATTEND_RING_CODEC, kernels-decode.ts:590-667)."""
    heads, L, S = 4, 2, 3
    ring = KvRing(layers=L, heads=heads, streams=S, capacity=capacity, dtype="f32", wrap=True)
    orc = oracle.Ring(layers=L, streams=S, heads=heads, capacity=capacity, dtype="f32", wrap=True)
    w = 3 * heads * HD
    rng = np.random.default_rng(capacity)
    # jump close to the wrap, then append across it
    first = capacity - 40
    for s in range(S):
        for layer in range(L):
            k = rng.standard_normal((heads, first, HD)).astype(np.float32)
            v = rng.standard_normal((heads, first, HD)).astype(np.float32)
            ring.ring_write(layer, s, 0, torch.from_numpy(k).to(DEV), torch.from_numpy(v).to(DEV))
            orc.kv_view()[layer, s, 0, :, :first] = k
            orc.kv_view()[layer, s, 1, :, :first] = v
            orc.slot_pos[layer, s, :first] = np.arange(first)
    worst = 0.0
    for step in range(first, capacity + 60):
        qkv = rng.standard_normal((S, w)).astype(np.float32)
        layer = step % L
        out = ring.append_attend(layer, [2, 0, 1], [step] * S, torch.from_numpy(qkv).to(DEV))
        ref, _ = orc.append_attend(layer, [2, 0, 1], [step] * S, qkv)
        worst = max(worst, max_err(out, ref))
    ring.sync()
    assert worst < TOL["f32"], worst
    last = capacity + 59
    for s in range(S):
        assert_window_equal(ring, orc, last % L, s, last % L, s, last)


@pytest.mark.parametrize("dtype,C,heads,wrap", [("f32", 17, 12, True), ("bf16", 32, 5, True), ("f16", 17, 5, True),
                                                ("bf16", 17, 12, False)])
def test_small_ring_parity(dtype, C, heads, wrap):
    """Rings of at most 32 slots (the local head's is 17) take the warp-per-head
    kernel: ring bytes and slot order bit-exact against the oracle, contexts
    within tolerance, fused == RoPE then attend bit for bit.  Streams at
    different positions, the ring wrapping several times; 5 heads leave idle
    warps in a CTA."""
    S, L = 3, 2
    qkv_w = 3 * heads * 64
    a = KvRing(layers=L, heads=heads, streams=S, capacity=C, dtype=dtype, wrap=wrap, max_position=256)
    b = KvRing(layers=L, heads=heads, streams=S, capacity=C, dtype=dtype, wrap=wrap, max_position=256)
    orc = oracle.Ring(layers=L, streams=S, heads=heads, capacity=C, dtype=dtype, wrap=wrap, max_position=256)
    start = [0, 3, 11]
    steps = 50 if wrap else C - max(start)
    worst = 0.0
    for step in range(steps):
        items = [2, 0, 1]
        pos = [step + start[s] for s in items]
        for layer in range(L):
            qkv = randn((S, qkv_w), seed=300 + step * 10 + layer)
            x = torch.from_numpy(qkv).to(DEV)
            oa = a.append_attend(layer, items, pos, x)
            qb = x.clone()
            b.rope_split_ring(layer, items, pos, qb)
            ob = b.attend_ring(layer, items, pos, qb, q_stride=qkv_w)
            assert torch.equal(oa, ob), (step, layer)
            ref, _ = orc.append_attend(layer, items, pos, qkv)
            worst = max(worst, max_err(oa, ref))
    a.sync()
    b.sync()
    assert worst < TOL[dtype], worst
    for layer in range(L):
        for s, p in zip(items, pos):
            assert_window_equal(a, orc, layer, s, layer, s, p)


@pytest.mark.parametrize("C", [17, 300])
def test_decode_on_a_capturing_stream(C):
    """Every launch goes to the caller's stream: append + attention captured into
    a CUDA graph on torch's capture stream and replayed (positions and rows
    updated in place between replays) gives, bit for bit, what the same calls
    give run directly -- for the small-ring kernel (C = 17) and the general one."""
    S = 3
    a = KvRing(layers=1, streams=S, capacity=C, dtype="bf16", wrap=True)
    b = KvRing(layers=1, streams=S, capacity=C, dtype="bf16", wrap=True)
    ids = torch.tensor([2, 0, 1], dtype=torch.int32, device=DEV)
    pos = torch.zeros(S, dtype=torch.int32, device=DEV)
    qkv = torch.zeros(S, QKV, device=DEV)
    out = torch.zeros(S, HID, device=DEV)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):  # one direct call before capturing (module loading)
        a.append_attend(0, ids, pos, qkv, out)
    torch.cuda.current_stream().wait_stream(side)
    a.reset()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        a.append_attend(0, ids, pos, qkv, out)
    for step in range(40):
        p = torch.tensor([step, step + 5, step + 9], dtype=torch.int32, device=DEV)
        x = torch.from_numpy(randn((S, QKV), seed=500 + step)).to(DEV)
        pos.copy_(p)
        qkv.copy_(x)
        g.replay()
        want = b.append_attend(0, ids, p, x)
        assert torch.equal(out, want), step
    torch.cuda.synchronize()
    a.sync()
    b.sync()
    del g


def test_bounded_wait_runs_out_and_the_context_recovers():
    """A decode whose chunk waits target a barrier that nothing signals (bounded
    at 20 000 cycles, ~10 us) gives up: mb_sync reports MB_ERR_TIMEOUT, the
    appends of that step are in the ring all the same (they precede the waits),
    and the next step at the default bound matches the oracle, which appended
    both steps."""
    S, C, L = 3, 200, 1
    ring = KvRing(layers=L, streams=S, capacity=C, dtype="f32", wrap=True)
    orc = oracle.Ring(layers=L, streams=S, heads=H, capacity=C, dtype="f32", wrap=True)
    items = [2, 0, 1]
    for step in range(150):  # windows of several chunks
        qkv = randn((S, QKV), seed=9000 + step)
        ring.append_attend(0, items, [step] * S, torch.from_numpy(qkv).to(DEV))
        orc.append_attend(0, items, [step] * S, qkv)
    ring.sync()
    ring.set_wait_limit(-20000)
    qkv = randn((S, QKV), seed=9150)
    ring.append_attend(0, items, [150] * S, torch.from_numpy(qkv).to(DEV))
    orc.append_attend(0, items, [150] * S, qkv)
    with pytest.raises(MockbirdError, match="MB_ERR_TIMEOUT"):
        ring.sync()
    ring.set_wait_limit(0)
    for s in items:
        assert_window_equal(ring, orc, 0, s, 0, s, 150)
    qkv = randn((S, QKV), seed=9151)
    out = ring.append_attend(0, items, [151] * S, torch.from_numpy(qkv).to(DEV))
    ref, _ = orc.append_attend(0, items, [151] * S, qkv)
    ring.sync()
    assert max_err(out, ref) < TOL["f32"]


@pytest.mark.parametrize("dtype,capacity", [("f32", 200), ("bf16", 300), ("f16", 24)])
def test_decode_step_equals_layer_by_layer(dtype, capacity):
    """mb_decode_step covers every layer in one launch (grid z = layer x item);
    its contexts and rings equal mb_append_attend called layer by layer, bit for
    bit, as windows grow past several split-K chunks and wrap (and on a ring of
    at most 32 slots, the warp-per-head path)."""
    S, L = 5, 4
    a = KvRing(layers=L, streams=S, capacity=capacity, dtype=dtype, wrap=True)
    b = KvRing(layers=L, streams=S, capacity=capacity, dtype=dtype, wrap=True)
    order = [3, 0, 4, 1]
    steps = capacity + 40
    for step in range(steps):
        qkv = torch.from_numpy(randn((L, len(order), QKV), seed=12000 + step)).to(DEV)
        pos = [step + 2 * i for i in range(len(order))]
        got = a.decode_step(order, pos, qkv)
        for layer in range(L):
            want = b.append_attend(layer, order, pos, qkv[layer].contiguous())
            assert torch.equal(got[layer], want), (step, layer)
    a.sync()
    b.sync()
    for layer in range(L):
        for s, p in zip(order, pos):
            ka, va, sa = a.gather(layer, s, p)
            kb, vb, sb = b.gather(layer, s, p)
            assert torch.equal(sa, sb) and torch.equal(ka, kb) and torch.equal(va, vb)
