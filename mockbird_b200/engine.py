"""Host-side mirror of the reference engine's KV-ring / attention interface.

The reference (liyu1981/mockbird, src/lib/tts/engine/) dispatches these WGSL
kernels from its runners; each method here is the same operation behind the
C ABI of include/mockbird_kv.h, with the same argument meaning and the same
error behaviour (a thrown error; the ring-overflow message is the one of
decode.ts:719-724):

    reference                                    here
    -------------------------------------------  ------------------------------
    ropeSplitRing / ropeSplitCodec dispatch      KvRing.rope_split_ring
      (decode.ts:527-535, codec.ts:593-624)
    attendRing / attendCodec dispatch            KvRing.attend_ring
      (decode.ts:536-552, codec.ts:626-645)
    the two in sequence, per layer               KvRing.append_attend  (one launch)
    DecodeRunner.globalStep's 12-layer loop      KvRing.decode_step (device arrays),
      (decode.ts:712-775)                          KvRing.decode_step_host (host arrays)
    PrefillRunner.run's rope/scores/softmax/     KvRing.prefill
      apply dispatches (prefill.ts:424-462)
    PrefillRunner.readLayerCache (:644-664)      KvRing.read_layer_cache
    PrefillRunner.poisonKv (:610-620)            KvRing.poison_kv
    WgpuTtsEngineImpl.reset / resetRings         KvRing.reset
      (gpu.ts:237-242, codec.ts:279-282)
    GpuTtsEngine.dispose (gpu.ts:283-291)        KvRing.dispose

Device tensors are torch CUDA tensors (device memory and streams only; the
arithmetic is in the CUDA library).  Calls run on torch's current stream of
the ring's device unless a stream is given.
"""
from __future__ import annotations

import ctypes
import numpy as np
import torch

from . import _lib

HD = 64


class MockbirdError(RuntimeError):
    """A non-zero mb_status from the library, with its message."""

    def __init__(self, code: int, message: str):
        self.code = code
        self.status = _lib.STATUS.get(code, str(code))
        super().__init__(f"{self.status}: {message}")


def _ptr(t) -> ctypes.c_void_p:
    if isinstance(t, torch.Tensor):
        return ctypes.c_void_p(t.data_ptr())
    if isinstance(t, np.ndarray):
        return ctypes.c_void_p(t.ctypes.data)
    raise TypeError(f"expected a torch tensor or numpy array, got {type(t).__name__}")


# The raw handle of a device's current CUDA stream: torch's C accessor where
# this torch has it (no Stream object per call), else the public API.
_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


_TORCH_DTYPE = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}


_NP_HOST = {"float32": np.dtype(np.float32), "int32": np.dtype(np.int32)}
_TORCH_HOST = {"float32": torch.float32, "int32": torch.int32}


def _host_array(name: str, a, shape: tuple, dtype: str):
    """Check a host buffer that the C ABI reads or writes in place through its
    address: a C-contiguous numpy array or CPU torch tensor of `dtype` and
    `shape` (anything else would be read or written at the wrong places)."""
    if isinstance(a, np.ndarray):
        ok = a.dtype == _NP_HOST[dtype] and a.shape == shape and a.flags.c_contiguous
    elif isinstance(a, torch.Tensor):
        ok = not a.is_cuda and a.dtype is _TORCH_HOST[dtype] and a.shape == shape and a.is_contiguous()
    else:
        ok = False
    if not ok:
        raise TypeError(f"{name} must be a contiguous host {dtype} array of shape {shape}")
    return a


def _host_addr(name: str, a, shape: tuple, dtype: str) -> int:
    """The address of a host buffer that passes _host_array."""
    _host_array(name, a, shape, dtype)
    return a.data_ptr() if isinstance(a, torch.Tensor) else a.ctypes.data


def _host_input(a):
    """An fp32 input read through its address: `a` itself when it is already a
    C-contiguous fp32 numpy array or CPU tensor, else a contiguous fp32 copy."""
    if isinstance(a, torch.Tensor) and not a.is_cuda:
        return a if a.dtype is torch.float32 and a.is_contiguous() else a.to(torch.float32).contiguous()
    if isinstance(a, np.ndarray) and a.dtype == _NP_HOST["float32"] and a.flags.c_contiguous:
        return a
    return np.ascontiguousarray(a, np.float32)


def _host_ids(streams, positions):
    """Stream ids and positions as int32 arrays of one length."""
    s = np.ascontiguousarray(streams, np.int32)
    p = np.ascontiguousarray(positions, np.int32)
    if s.ndim != 1 or p.shape != s.shape:
        raise ValueError(f"streams and positions must be 1-D of one length (got {s.shape} and {p.shape})")
    return s, p


class KvRing:
    """The rings of `streams` independent synthesis streams on one GPU.

    Geometry (mb_config): kv[layer][stream][K|V][head][slot][64] in `dtype`,
    slot_pos[layer][stream][slot].  `wrap=False` is the reference's global ring
    (positions must stay below `capacity`), `wrap=True` its codec ring
    (slot = position % capacity).
    """

    def __init__(self, layers: int = 12, heads: int = 12, capacity: int = 570, streams: int = 1,
                 dtype: str = "f32", wrap: bool = False, max_position: int = 65536,
                 rope_theta: float = 10000.0, device: int = 0, max_batch: int = 0):
        self.lib = _lib.load()
        if dtype not in _lib.DTYPES:
            raise ValueError(f"dtype must be one of {sorted(_lib.DTYPES)}")
        cfg = _lib.MbConfig()
        self.lib.mb_config_default(ctypes.byref(cfg))
        cfg.layers, cfg.heads, cfg.head_dim, cfg.capacity = layers, heads, HD, capacity
        cfg.streams, cfg.dtype, cfg.wrap = streams, _lib.DTYPES[dtype], int(bool(wrap))
        cfg.max_position, cfg.rope_theta, cfg.device, cfg.max_batch = max_position, rope_theta, device, max_batch
        handle = ctypes.c_void_p()
        rc = self.lib.mb_create(ctypes.byref(cfg), ctypes.byref(handle))
        if rc:
            raise MockbirdError(rc, f"mb_create failed (layers={layers} heads={heads} capacity={capacity} "
                                    f"streams={streams} dtype={dtype} device={device})")
        self.ctx = handle
        self.layers, self.heads, self.capacity, self.streams = layers, heads, capacity, streams
        self.dtype, self.wrap, self.device = dtype, bool(wrap), torch.device("cuda", device)
        self.max_position = max_position
        self.max_batch = max_batch or streams
        self.hidden = heads * HD
        self.torch_dtype = _TORCH_DTYPE[dtype]

    # ------------------------------------------------------------ plumbing
    def _check(self, rc: int) -> None:
        if rc:
            raise MockbirdError(rc, self.lib.mb_last_error(self.ctx).decode())

    def _stream(self, stream) -> ctypes.c_void_p:
        if stream is None:
            if _raw_stream is not None:
                return ctypes.c_void_p(_raw_stream(self.device.index))
            stream = torch.cuda.current_stream(self.device)
        return ctypes.c_void_p(stream.cuda_stream if isinstance(stream, torch.cuda.Stream) else int(stream))

    def _ids(self, values) -> torch.Tensor:
        if isinstance(values, torch.Tensor) and values.is_cuda:
            if values.dtype != torch.int32 or not values.is_contiguous():
                raise TypeError("stream ids / positions must be a contiguous int32 tensor")
            return values
        return torch.as_tensor(np.asarray(values, dtype=np.int32), device=self.device)

    def _dev(self, t: torch.Tensor, dtype=torch.float32) -> torch.Tensor:
        if not (isinstance(t, torch.Tensor) and t.is_cuda and t.dtype == dtype and t.is_contiguous()):
            raise TypeError(f"expected a contiguous CUDA {dtype} tensor")
        return t

    @property
    def info(self) -> _lib.MbRingInfo:
        out = _lib.MbRingInfo()
        self._check(self.lib.mb_ring_info_get(self.ctx, ctypes.byref(out)))
        return out

    # ------------------------------------------------------------ decode
    def rope_split_ring(self, layer: int, streams, positions, qkv: torch.Tensor, stream=None) -> torch.Tensor:
        """ROPE_SPLIT_RING / _CODEC: Q roped in place in `qkv` [n][3*H*64]; K/V appended."""
        s, p, q = self._ids(streams), self._ids(positions), self._dev(qkv)
        self._check(self.lib.mb_rope_append(self.ctx, layer, s.numel(), _ptr(s), _ptr(p), _ptr(q),
                                             self._stream(stream)))
        return qkv

    def attend_ring(self, layer: int, streams, positions, q: torch.Tensor, out: torch.Tensor | None = None,
                    q_stride: int | None = None, stream=None) -> torch.Tensor:
        """ATTEND_RING / _CODEC: roped queries (row stride q_stride) -> context [n][H*64]."""
        s, p, qq = self._ids(streams), self._ids(positions), self._dev(q)
        n = s.numel()
        stride = q_stride if q_stride is not None else qq.shape[-1]
        if out is None:
            out = torch.empty(n, self.hidden, dtype=torch.float32, device=self.device)
        self._check(self.lib.mb_attend(self.ctx, layer, n, _ptr(s), _ptr(p), _ptr(qq), stride, _ptr(self._dev(out)),
                                       self._stream(stream)))
        return out

    def append_attend(self, layer: int, streams, positions, qkv: torch.Tensor, out: torch.Tensor | None = None,
                      stream=None) -> torch.Tensor:
        """The fused hot path: append + RoPE + attention for n streams of one layer."""
        s, p, q = self._ids(streams), self._ids(positions), self._dev(qkv)
        n = s.numel()
        if out is None:
            out = torch.empty(n, self.hidden, dtype=torch.float32, device=self.device)
        self._check(self.lib.mb_append_attend(self.ctx, layer, n, _ptr(s), _ptr(p), _ptr(q), _ptr(self._dev(out)),
                                              self._stream(stream)))
        return out

    def decode_step(self, streams, positions, qkv: torch.Tensor, out: torch.Tensor | None = None,
                    stream=None) -> torch.Tensor:
        """All layers of one decode step on device: qkv [layers][n][3*H*64] -> [layers][n][H*64]."""
        s, p, q = self._ids(streams), self._ids(positions), self._dev(qkv)
        n = s.numel()
        if out is None:
            out = torch.empty(self.layers, n, self.hidden, dtype=torch.float32, device=self.device)
        self._check(self.lib.mb_decode_step(self.ctx, n, _ptr(s), _ptr(p), _ptr(q), _ptr(self._dev(out)),
                                            self._stream(stream)))
        return out

    def append_attend_host(self, layer: int, streams, positions, qkv: np.ndarray,
                           out: np.ndarray | None = None, stream=None) -> np.ndarray:
        """append_attend on host arrays (validated on the host; blocks until `out` is ready).

        `qkv` / `out` may be numpy arrays or (pinned) CPU torch tensors."""
        s, p = _host_ids(streams, positions)
        n = len(s)
        q = _host_input(qkv)
        if out is None:
            out = np.empty((n, self.hidden), np.float32)
        qa = _host_addr("qkv", q, (n, 3 * self.hidden), "float32")
        oa = _host_addr("out", out, (n, self.hidden), "float32")
        self._check(self.lib.mb_append_attend_host(self.ctx, layer, n, s.ctypes.data, p.ctypes.data, qa, oa,
                                                   self._stream(stream)))
        return out

    def decode_step_host(self, streams, positions, qkv, out=None, stream=None):
        """All layers of one decode step on host buffers: qkv [layers][n][3*H*64] -> [layers][n][H*64].

        `qkv` / `out` may be numpy arrays or (pinned) CPU torch tensors."""
        s, p = _host_ids(streams, positions)
        n = len(s)
        q = _host_input(qkv)
        if out is None:
            out = np.empty((self.layers, n, self.hidden), np.float32)
        qa = _host_addr("qkv", q, (self.layers, n, 3 * self.hidden), "float32")
        oa = _host_addr("out", out, (self.layers, n, self.hidden), "float32")
        self._check(self.lib.mb_decode_step_host(self.ctx, n, s.ctypes.data, p.ctypes.data, qa, oa,
                                                 self._stream(stream)))
        return out

    # ------------------------------------------------------------ prefill
    def prefill(self, layer: int, streams, qkv: torch.Tensor, out: torch.Tensor | None = None,
                stream=None) -> torch.Tensor:
        """Causal prefill of positions 0..rows-1: qkv [n][rows][3*H*64] -> context [n][rows][H*64]."""
        s, q = self._ids(streams), self._dev(qkv)
        n, rows = q.shape[0], q.shape[1]
        if out is None:
            out = torch.empty(n, rows, self.hidden, dtype=torch.float32, device=self.device)
        self._check(self.lib.mb_prefill(self.ctx, layer, n, _ptr(s), rows, _ptr(q), _ptr(self._dev(out)),
                                        self._stream(stream)))
        return out

    # ------------------------------------------------------------ cache access
    def gather(self, layer: int, stream_id: int, position: int, stream=None):
        """Live window in position order: (k [H][W][64], v, slots [W]) device tensors, storage dtype."""
        W = min(position + 1, self.capacity)
        k = torch.empty(self.heads, W, HD, dtype=self.torch_dtype, device=self.device)
        v = torch.empty_like(k)
        slots = torch.empty(W, dtype=torch.int32, device=self.device)
        self._check(self.lib.mb_gather(self.ctx, layer, stream_id, position, _ptr(k), _ptr(v), _ptr(slots),
                                       self._stream(stream)))
        return k, v, slots

    def read_layer_cache(self, layer: int, stream_id: int, rows: int, stream=None):
        """PrefillRunner.readLayerCache: K and V of positions 0..rows-1 as [rows][H*64] f32."""
        k, v, _ = self.gather(layer, stream_id, rows - 1, stream)
        return (k.float().permute(1, 0, 2).reshape(-1, self.hidden),
                v.float().permute(1, 0, 2).reshape(-1, self.hidden))

    def ring_write(self, layer: int, stream_id: int, first_position: int, k: torch.Tensor, v: torch.Tensor,
                   stream=None) -> None:
        """Write K (already roped) / V rows [H][count][64] (storage dtype) at positions first_position.."""
        k, v = self._dev(k, self.torch_dtype), self._dev(v, self.torch_dtype)
        self._check(self.lib.mb_ring_write(self.ctx, layer, stream_id, first_position, k.shape[1], _ptr(k), _ptr(v),
                                           self._stream(stream)))

    def poison_kv(self, layer: int, stream_id: int, rows: int, value: float = -12345.5, stream=None) -> None:
        """PrefillRunner.poisonKv: write a sentinel into positions 0..rows-1."""
        k = torch.full((self.heads, rows, HD), value, dtype=self.torch_dtype, device=self.device)
        self.ring_write(layer, stream_id, 0, k, k.clone(), stream)

    def reset(self, stream_id: int = -1, stream=None) -> None:
        """Every slot of `stream_id` (all streams if -1) becomes empty."""
        self._check(self.lib.mb_reset(self.ctx, stream_id, self._stream(stream)))

    def set_wait_limit(self, cycles: int) -> None:
        """Bound (SM cycles) of the decode kernels' waits for their K/V chunks;
        0 restores the default (about 2 s).  A wait that runs out surfaces as
        MB_ERR_TIMEOUT at the next sync.  Negative: every wait targets a barrier
        that nothing signals and runs out after -cycles (the test of that path)."""
        self._check(self.lib.mb_set_wait_limit(self.ctx, int(cycles)))

    def sync(self, stream=None) -> None:
        """Wait for the stream and raise on any device-side rejection."""
        self._check(self.lib.mb_sync(self.ctx, self._stream(stream)))

    def dispose(self) -> None:
        if getattr(self, "ctx", None):
            self.lib.mb_destroy(self.ctx)
            self.ctx = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.dispose()

    def __del__(self):
        try:
            self.dispose()
        except Exception:
            pass



class Decoder:
    """The global decode step around the ring, mirroring
    DecodeRunner.globalStep (decode.ts:712-775) without the embedding: every layer
    LN1 -> QKV -> append + RoPE + attention -> c_proj + residual -> LN2 -> fc_in ->
    GELU(tanh) -> fc_out + residual, then ln_f, for n streams at once.

    `weights`: one fp32 array in the published graph's order (see
    mb_decoder_weight_count / mb_decoder_create in include/mockbird_kv.h)."""

    def __init__(self, ring: KvRing, weights: np.ndarray, ffn: int = 3072):
        self.ring, self.lib, self.ffn = ring, ring.lib, ffn
        w = np.ascontiguousarray(weights, np.float32)
        want = self.lib.mb_decoder_weight_count(ring.ctx, ffn)
        if w.size != want:
            raise ValueError(f"decoder weights: {w.size} values, expected {want}")
        handle = ctypes.c_void_p()
        ring._check(self.lib.mb_decoder_create(ring.ctx, ffn, _ptr(w), w.size, ctypes.byref(handle)))
        self.handle = handle

    @staticmethod
    def weight_count(layers: int, hidden: int, ffn: int) -> int:
        h, f = hidden, ffn
        return layers * (2 * h + h * 3 * h + 3 * h + h * h + h + 2 * h + h * f + f + f * h + h) + 2 * h

    def step(self, streams, positions, hidden: torch.Tensor, stream=None) -> torch.Tensor:
        """hidden [n][H*64] fp32 (device): embedded rows in, ln_f output out (in place)."""
        s, p, x = self.ring._ids(streams), self.ring._ids(positions), self.ring._dev(hidden)
        rc = self.lib.mb_decoder_step(self.handle, s.numel(), _ptr(s), _ptr(p), _ptr(x), self.ring._stream(stream))
        if rc:
            raise MockbirdError(rc, self.lib.mb_last_error(self.ring.ctx).decode())
        return hidden

    def step_host(self, streams, positions, hidden, stream=None):
        """One step on host arrays, as DecodeRunner.globalStep (decode.ts:712-775)
        writes the embedded row and reads back ln_f: hidden [n][H*64] fp32 (numpy
        or a CPU tensor, ideally pinned) is updated in place; blocks until done."""
        s = np.ascontiguousarray(streams, np.int32)
        p = np.ascontiguousarray(positions, np.int32)
        if len(p) != len(s):
            raise ValueError("streams and positions differ in length")
        _host_array("hidden", hidden, (len(s), self.ring.hidden), "float32")
        rc = self.lib.mb_decoder_step_host(self.handle, len(s), _ptr(s), _ptr(p), _ptr(hidden),
                                           self.ring._stream(stream))
        if rc:
            raise MockbirdError(rc, self.lib.mb_last_error(self.ring.ctx).decode())
        return hidden

    def dispose(self) -> None:
        if getattr(self, "handle", None):
            self.lib.mb_decoder_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.dispose()
        except Exception:
            pass


class LocalHead:
    """The local 17-step head (DecodeRunner.nextFrame, decode.ts:788-939) for n
    streams at once: one frame of `channels` audio codes per stream plus the
    continue/stop decision, the repetition-penalty seen masks kept on the device
    (clearSeen, decode.ts:275-280, is `clear`).

    `ring`: the local ring -- a KvRing with one layer and capacity >= channels + 1.
    `weights`: one fp32 array in the order of mb_local_head_create
    (include/mockbird_kv.h); `weight_count` gives its length."""

    def __init__(self, ring: KvRing, weights: np.ndarray, ffn: int = 3072, codes: int = 1024,
                 channels: int = 16, repetition_penalty: float = 1.2):
        self.ring, self.lib = ring, ring.lib
        self.ffn, self.codes, self.channels, self.penalty = ffn, codes, channels, repetition_penalty
        self.cfg = _lib.MbLocalConfig(ffn, codes, channels, repetition_penalty)
        w = np.ascontiguousarray(weights, np.float32)
        want = self.lib.mb_local_head_weight_count(ring.ctx, ctypes.byref(self.cfg))
        if want and w.size != want:  # 0: the ring does not suit; create reports why
            raise ValueError(f"local head weights: {w.size} values, expected {want}")
        handle = ctypes.c_void_p()
        ring._check(self.lib.mb_local_head_create(ring.ctx, ctypes.byref(self.cfg), _ptr(w), w.size,
                                                  ctypes.byref(handle)))
        self.handle = handle

    @staticmethod
    def weight_count(hidden: int, ffn: int, codes: int, channels: int) -> int:
        h = hidden
        return Decoder.weight_count(1, h, ffn) + h + 2 * h + (channels - 1) * codes * h + channels * h * codes

    def clear(self, stream: int = -1, cuda_stream=None) -> None:
        """Zero the seen masks of `stream` (all streams when -1): a new utterance."""
        self.ring._check(self.lib.mb_local_head_clear(self.handle, int(stream), self.ring._stream(cuda_stream)))

    def frame(self, streams, hidden: torch.Tensor, logits: bool = False, stream=None):
        """hidden [n][H*64] fp32 (device): the global step's ln_f output.

        Returns (tokens [n][channels] int32, cont [n] int32 -- 1 continue, 0 stop,
        logits [n][channels][codes] fp32 before the penalty, or None)."""
        s, x = self.ring._ids(streams), self.ring._dev(hidden)
        n = s.numel()
        tok = torch.empty(n, self.channels, dtype=torch.int32, device=self.ring.device)
        cont = torch.empty(n, dtype=torch.int32, device=self.ring.device)
        lg = (torch.empty(n, self.channels, self.codes, dtype=torch.float32, device=self.ring.device)
              if logits else None)
        rc = self.lib.mb_local_head_frame(self.handle, n, _ptr(s), _ptr(x), _ptr(tok), _ptr(cont),
                                          _ptr(lg) if lg is not None else None, self.ring._stream(stream))
        self.ring._check(rc)
        return tok, cont, lg

    def frame_host(self, streams, hidden, tokens=None, cont=None, stream=None):
        """One frame on host arrays, as nextFrame (decode.ts:788-939) takes the
        hidden row from the host and reads its tokens back: hidden [n][H*64] fp32
        (numpy or a CPU tensor, ideally pinned).  Blocks until the outputs are in
        place.  Returns (tokens [n][channels] int32, cont [n] int32)."""
        s = np.ascontiguousarray(streams, np.int32)
        if isinstance(hidden, np.ndarray):
            hidden = np.ascontiguousarray(hidden, np.float32)
        n = len(s)
        if tokens is None:
            tokens = np.empty((n, self.channels), np.int32)
        if cont is None:
            cont = np.empty(n, np.int32)
        _host_array("hidden", hidden, (n, self.ring.hidden), "float32")
        _host_array("tokens", tokens, (n, self.channels), "int32")
        _host_array("cont", cont, (n,), "int32")
        rc = self.lib.mb_local_head_frame_host(self.handle, n, _ptr(s), _ptr(hidden), _ptr(tokens), _ptr(cont),
                                               self.ring._stream(stream))
        self.ring._check(rc)
        return tokens, cont

    def dispose(self) -> None:
        if getattr(self, "handle", None):
            self.lib.mb_local_head_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.dispose()
        except Exception:
            pass


def argmax_penalty(logits: torch.Tensor, seen: torch.Tensor, penalty: float, stream=None) -> torch.Tensor:
    """ARGMAX_PENALTY (kernels-decode.ts:428-485) on the device: per row of
    logits [n][codes] fp32, the penalised argmax under seen [n][codes/32] (int32
    words holding the mask bits), whose bit is then set in place.  Returns the
    ids [n] int32."""
    lib = _lib.load()
    if not (logits.is_cuda and logits.dtype == torch.float32 and logits.is_contiguous() and logits.dim() == 2):
        raise TypeError("logits must be a contiguous 2-D CUDA float32 tensor")
    n, codes = logits.shape
    if not (seen.is_cuda and seen.dtype == torch.int32 and seen.is_contiguous() and seen.shape == (n, codes // 32)):
        raise TypeError("seen must be a contiguous CUDA int32 tensor [n][codes/32]")
    out = torch.empty(n, dtype=torch.int32, device=logits.device)
    if stream is None:
        stream = torch.cuda.current_stream(logits.device)
    with torch.cuda.device(logits.device):
        rc = lib.mb_argmax_penalty(n, codes, _ptr(logits), _ptr(seen), penalty, _ptr(out),
                                   ctypes.c_void_p(stream.cuda_stream))
    if rc:
        raise MockbirdError(rc, "mb_argmax_penalty: bad arguments or launch failure")
    return out
