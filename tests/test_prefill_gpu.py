"""GPU parity of the causal prefill (ROPE_SPLIT_CACHE + causal attention) through
the C ABI, against the CPU oracle."""
import numpy as np
import pytest
import torch

import oracle
from gpu_util import HID, QKV, TOL, H, assert_window_equal, max_err, randn
from mockbird_b200 import KvRing, MockbirdError

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _prefill_both(dtype, streams, rows, capacity, n_streams, seed, scale=1.0, layer=0, layers=1):
    ring = KvRing(layers=layers, streams=n_streams, capacity=capacity, dtype=dtype, wrap=True)
    orc = oracle.Ring(layers=layers, streams=n_streams, heads=H, capacity=capacity, dtype=dtype, wrap=True)
    qkv = randn((len(streams), rows, QKV), seed=seed, scale=scale)
    out = ring.prefill(layer, streams, torch.from_numpy(qkv).to(DEV))
    ref, _ = orc.prefill(layer, streams, qkv, q_round=(dtype != "f32"))
    return ring, orc, out, ref


def test_prefill_f32_195_rows():
    """The golden prompt's shape (195 rows), fp32 ring of 570 slots (gpu.ts:362)."""
    ring, orc, out, ref = _prefill_both("f32", [1, 0], 195, 570, 2, seed=11)
    ring.sync()
    assert max_err(out, ref) < TOL["f32"]
    for s in (0, 1):
        assert_window_equal(ring, orc, 0, s, 0, s, 194)


@pytest.mark.parametrize("dtype", ["f16", "bf16", "f32"])
def test_prefill_444_rows(dtype):
    """BASELINE config 3's shape: 188-frame prompt + 256 text = 444 positions,
    q/k/v ~ N(0, 0.5), 16-bit storage with fp32 accumulation (and the fp32 ring,
    attended over bf16 hi/lo operand parts), ring capacity 2048."""
    ring, orc, out, ref = _prefill_both(dtype, [3, 0, 2], 444, 2048, 4, seed=12, scale=0.5)
    ring.sync()
    assert max_err(out, ref) < TOL[dtype]
    for s in (0, 2, 3):
        assert_window_equal(ring, orc, 0, s, 0, s, 443)


def test_prefill_config3_full_batch():
    """BASELINE config 3 at its batch: 32 streams x 444 rows in one call (1 536
    attention CTAs, several waves of them), fp16 ring of 2048 slots, q/k/v ~
    N(0, 0.5); every context row against the oracle, windows bit-exact for a
    sample of streams."""
    ring, orc, out, ref = _prefill_both("f16", list(range(32)), 444, 2048, 32, seed=33, scale=0.5)
    ring.sync()
    assert max_err(out, ref) < TOL["f16"]
    for s in (0, 17, 31):
        assert_window_equal(ring, orc, 0, s, 0, s, 443)


@pytest.mark.parametrize("dtype", ["f16", "f32"])
@pytest.mark.parametrize("rows", [1, 2, 63, 64, 65, 128, 191, 257, 300])
def test_prefill_row_edges(rows, dtype):
    """Tile edges of both attention kernels: 128-query / 64-key tiles on tensor
    cores (16-bit rings; the fp32 ring over bf16 hi/lo operand parts).  Query
    tiles are laid out from the last row back, so the partial tile is the first
    (rows 191, 257 and 300 leave 63, 1 and 44 rows in it)."""
    ring, orc, out, ref = _prefill_both(dtype, [0], rows, 300, 1, seed=rows, scale=0.5)
    ring.sync()
    assert max_err(out, ref) < TOL[dtype]
    assert_window_equal(ring, orc, 0, 0, 0, 0, rows - 1)


def test_prefill_at_full_capacity_then_decode_wraps():
    ring, orc, out, ref = _prefill_both("f32", [0], 256, 256, 1, seed=5)
    assert max_err(out, ref) < TOL["f32"]
    for step in range(256, 300):  # the first decode steps already wrap
        qkv = randn((1, QKV), seed=step)
        o = ring.append_attend(0, [0], [step], torch.from_numpy(qkv).to(DEV))
        r, _ = orc.append_attend(0, [0], [step], qkv)
        assert max_err(o, r) < TOL["f32"]
    ring.sync()
    assert_window_equal(ring, orc, 0, 0, 0, 0, 299)


def test_prefill_starts_an_utterance():
    """A prefill over a used ring marks the old slots empty: the next decode step
    attends positions 0..rows only (the per-chunk reset of runtime.ts:520-523)."""
    C = 64
    ring = KvRing(layers=1, streams=1, capacity=C, dtype="f32", wrap=True)
    orc = oracle.Ring(layers=1, streams=1, heads=H, capacity=C, dtype="f32", wrap=True)
    for step in range(100):  # an earlier utterance that wrapped
        qkv = randn((1, QKV), seed=step)
        ring.append_attend(0, [0], [step], torch.from_numpy(qkv).to(DEV))
        orc.append_attend(0, [0], [step], qkv)
    qkv = randn((1, 20, QKV), seed=500)
    out = ring.prefill(0, [0], torch.from_numpy(qkv).to(DEV))
    orc.reset(0)
    ref, _ = orc.prefill(0, [0], qkv)
    assert max_err(out, ref) < TOL["f32"]
    q = randn((1, QKV), seed=501)
    o = ring.append_attend(0, [0], [20], torch.from_numpy(q).to(DEV))
    r, _ = orc.append_attend(0, [0], [20], q)
    ring.sync()
    assert max_err(o, r) < TOL["f32"]
    assert_window_equal(ring, orc, 0, 0, 0, 0, 20)


def test_prefill_errors():
    ring = KvRing(layers=2, streams=2, capacity=32, dtype="f16", wrap=True)
    qkv = torch.zeros(1, 33, QKV, device=DEV)
    with pytest.raises(MockbirdError) as e:
        ring.prefill(0, [0], qkv)
    assert e.value.status == "MB_ERR_CAPACITY"
    with pytest.raises(MockbirdError) as e:
        ring.prefill(2, [0], qkv[:, :4].contiguous())
    assert e.value.status == "MB_ERR_LAYER"
    out = ring.prefill(1, torch.tensor([5], dtype=torch.int32, device=DEV), qkv[:, :4].contiguous())
    with pytest.raises(MockbirdError) as e:
        ring.sync()
    assert e.value.status == "MB_ERR_DEVICE"
    del out
    ring.sync()


@pytest.mark.parametrize("dtype", ["f16", "f32"])
def test_prefill_skips_rejected_items(dtype):
    """A call whose first item names a stream the ring does not have: that item is
    rejected on the device (MB_ERR_DEVICE at the next sync), and the other items
    of the same call still match the oracle -- the persistent attention CTAs skip
    the rejected item's query tiles (for some CTAs their first work item) and
    carry on with the next ones."""
    rows = 200
    ring = KvRing(layers=1, streams=3, capacity=256, dtype=dtype, wrap=True)
    orc = oracle.Ring(layers=1, streams=3, heads=H, capacity=256, dtype=dtype, wrap=True)
    qkv = randn((3, rows, QKV), seed=41, scale=0.5)
    ids = torch.tensor([7, 0, 2], dtype=torch.int32, device=DEV)  # no stream 7
    out = ring.prefill(0, ids, torch.from_numpy(qkv).to(DEV))
    with pytest.raises(MockbirdError) as e:
        ring.sync()
    assert e.value.status == "MB_ERR_DEVICE"
    ref, _ = orc.prefill(0, [0, 2], qkv[1:], q_round=(dtype != "f32"))
    assert max_err(out[1:], ref) < TOL[dtype]
    for s in (0, 2):
        assert_window_equal(ring, orc, 0, s, 0, s, rows - 1)


@pytest.mark.parametrize("dtype", ["f16", "bf16", "f32"])
def test_prefill_rising_scores_rescale_every_tile(dtype):
    """Scores that rise along the keys, so that every row's running maximum jumps
    by more than 2^8 (log2 units) on every 64-key tile: the tensor-core kernel
    then rescales the row's O in tensor memory on every tile.  Q and K put their
    energy into the last RoPE pair of each head (frequency 10000^(-62/64): it
    turns by less than 0.2 rad over the 1000 positions), K growing with the
    position, so q.k grows by ~9 per tile after the 0.125 * log2(e) scale.
    1000 rows: 8 query tiles of 128, up to 16 key tiles.  Also the longest
    prefill of the suite.  Random V."""
    rows, C = 1000, 1024
    ring = KvRing(layers=1, streams=1, capacity=C, dtype=dtype, wrap=True)
    orc = oracle.Ring(layers=1, streams=1, heads=H, capacity=C, dtype=dtype, wrap=True)
    rng = np.random.default_rng(31)
    qkv = np.zeros((1, rows, QKV), np.float32)
    for h in range(H):
        qkv[0, :, h * 64 + 62: h * 64 + 64] = 4.0                                  # q
        qkv[0, :, HID + h * 64 + 62: HID + h * 64 + 64] = (0.1 * np.arange(rows))[:, None]  # k
    qkv[0, :, 2 * HID:] = rng.standard_normal((rows, HID)).astype(np.float32)      # v
    out = ring.prefill(0, [0], torch.from_numpy(qkv).to(DEV))
    ref, _ = orc.prefill(0, [0], qkv, q_round=(dtype != "f32"))
    ring.sync()
    assert max_err(out, ref) < TOL[dtype]
    assert_window_equal(ring, orc, 0, 0, 0, 0, rows - 1)
