"""GPU test of mb_append_attend_noalloc, the decode entry point for callers that
cannot allocate device memory (their memory belongs to another allocator, or
they run on a thread that must not block on cudaMalloc).

The test plays such a caller: it owns the ring, the RoPE table, the inputs, the
outputs and the status word (allocated here by torch, as a host framework
would), and calls the entry point through the C ABI.  Its results must match
the allocating entry point, mb_append_attend, on two calls in a row whose
windows span several split-K chunks, i.e. whose partials go through the
library's fixed scratch array.  Collected last, so that a run stopping at the
first failure has run every other test first; it also passes alone.
"""
import ctypes

import numpy as np
import pytest
import torch

from mockbird_b200 import KvRing, _lib

pytestmark = pytest.mark.gpu

H, HD = 12, 64
QKV = 3 * H * HD
TOL = {"f32": 2e-3, "bf16": 1e-2, "f16": 1e-2}  # the attention tolerances every decode test uses
TORCH = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}
CODE = {"f32": _lib.MB_F32, "bf16": _lib.MB_BF16, "f16": _lib.MB_F16}


def _rope_table(max_position, theta=10000.0):
    """The documented table: fp64 angle and cos/sin, rounded once to fp32."""
    inv = theta ** (-(2.0 * np.arange(32)) / 64.0)
    ang = np.arange(max_position, dtype=np.float64)[:, None] * inv[None, :]
    return np.stack([np.cos(ang), np.sin(ang)], -1).astype(np.float32)  # [P][32][2]


# capacity 300: windows of 4 fp32 / 2 16-bit split-K chunks, whose partials go
# through the fixed scratch array; capacity 17: the warp-per-head path of rings
# of at most 32 slots (no split-K), wrapping on the second call
@pytest.mark.parametrize("dtype,capacity,filled", [("f32", 300, 250), ("bf16", 300, 250), ("f16", 300, 250),
                                                   ("f32", 17, 16), ("bf16", 17, 16)])
def test_noalloc_matches_the_allocating_entry_point(dtype, capacity, filled):
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    L, S, C, P = 2, 4, capacity, 4096
    td = TORCH[dtype]
    ref = KvRing(layers=L, streams=S, capacity=C, dtype=dtype, wrap=True, max_position=P)

    # caller-owned ring, laid out like a context's
    kv = torch.zeros(L, S, 2, H, C, HD, dtype=td, device=dev)
    slot_pos = torch.full((L, S, C), -1, dtype=torch.int32, device=dev)
    rope = torch.from_numpy(_rope_table(P)).to(dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    ring = _lib.MbRingRef(kv.data_ptr(), slot_pos.data_ptr(), rope.data_ptr(), status.data_ptr(),
                          L, H, C, S, CODE[dtype], 1, P)

    # the same earlier positions in both rings
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    for layer in range(L):
        for s in range(S):
            k = torch.randn(H, filled, HD, generator=g, device=dev).to(td)
            v = torch.randn(H, filled, HD, generator=g, device=dev).to(td)
            ref.ring_write(layer, s, 0, k, v)
            kv[layer, s, 0, :, :filled] = k
            kv[layer, s, 1, :, :filled] = v
            slot_pos[layer, s, :filled] = torch.arange(filled, dtype=torch.int32, device=dev)

    items = torch.tensor([2, 0, 3], dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev)
    for step in (filled, filled + 1):  # two calls in a row
        pos = torch.full((3,), step, dtype=torch.int32, device=dev)
        qkv = torch.randn(3, QKV, generator=g, device=dev)
        want = ref.append_attend(1, items, pos, qkv)
        got = torch.empty(3, H * HD, dtype=torch.float32, device=dev)
        rc = lib.mb_append_attend_noalloc(ctypes.byref(ring), 1, 3, ctypes.c_void_p(items.data_ptr()),
                                          ctypes.c_void_p(pos.data_ptr()), ctypes.c_void_p(qkv.data_ptr()),
                                          ctypes.c_void_p(got.data_ptr()), ctypes.c_void_p(stream.cuda_stream))
        assert rc == 0
        torch.cuda.synchronize(dev)
        assert float((got - want).abs().max()) < TOL[dtype]
        # the appended rows and positions agree bit for bit: both calls rope the
        # same row with the same table values
        k_ref, v_ref, slots_ref = ref.gather(1, 2, step)
        W = min(step + 1, C)
        assert torch.equal(slot_pos[1, 2][slots_ref.long()],
                           torch.arange(step - W + 1, step + 1, device=dev, dtype=torch.int32))
        assert torch.equal(kv[1, 2, 0, :, step % C], k_ref[:, -1])
        assert torch.equal(kv[1, 2, 1, :, step % C], v_ref[:, -1])
    ref.sync()
    assert int(status.item()) == 0


def test_noalloc_rejects_calls_beyond_its_scratch():
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    buf = torch.zeros(64, dtype=torch.int32, device=dev)
    p = buf.data_ptr()
    # 64 streams x 12 heads x ceil(1_000_000 / 64) chunks of partials: far beyond the fixed array
    ring = _lib.MbRingRef(p, p, p, p, 1, H, 1_000_000, 64, _lib.MB_F32, 1, 1 << 20)
    assert lib.mb_append_attend_noalloc(ctypes.byref(ring), 0, 64, p, p, p, p, None) == 1  # MB_ERR_ARG
    ring.rope = None
    assert lib.mb_append_attend_noalloc(ctypes.byref(ring), 0, 1, p, p, p, p, None) == 1
