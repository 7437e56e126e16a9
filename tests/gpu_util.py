"""Helpers shared by the GPU parity tests (CUDA side vs the CPU oracle)."""
import numpy as np
import torch

import oracle

H, HD = 12, 64
HID = H * HD
QKV = 3 * HID
# attention tolerances from the task statement: max-abs 2e-3 with fp32 storage,
# 1e-2 with fp16/bf16 storage
TOL = {"f32": 2e-3, "bf16": 1e-2, "f16": 1e-2}
TORCH_DT = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}


def to_np_storage(t: torch.Tensor) -> np.ndarray:
    """Device tensor in the storage dtype -> numpy with the oracle's representation
    (float32, or uint16 bit patterns for 16-bit storage)."""
    if t.dtype == torch.float32:
        return t.cpu().numpy()
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


def from_np_storage(a: np.ndarray, dtype: str, device="cuda") -> torch.Tensor:
    if dtype == "f32":
        return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(device)
    t = torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).to(device)
    return t.view(TORCH_DT[dtype])


def assert_window_equal(ring, orc, layer, stream, orc_layer, orc_stream, position):
    """Gathered window (K/V bytes, slot indices, wrap order) bit-exact vs the oracle."""
    k, v, slots = ring.gather(layer, stream, position)
    ok, ov, oslots = orc.gather(orc_layer, orc_stream, position)
    assert np.array_equal(slots.cpu().numpy(), oslots), (layer, stream, position)
    assert np.array_equal(to_np_storage(k), ok), (layer, stream, position)
    assert np.array_equal(to_np_storage(v), ov), (layer, stream, position)


def max_err(a, b) -> float:
    a = a.detach().cpu().numpy() if isinstance(a, torch.Tensor) else a
    b = b.detach().cpu().numpy() if isinstance(b, torch.Tensor) else b
    return float(np.abs(a.astype(np.float64) - b.astype(np.float64)).max()) if np.size(a) else 0.0


def randn(shape, seed, scale=1.0):
    return (np.random.default_rng(seed).standard_normal(shape) * scale).astype(np.float32)


def oracle_ring(**kw):
    return oracle.Ring(**kw)
