"""CPU oracle for the KV-ring / RoPE / attention path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
(and its ``--impl reference`` arm) may import this package.  It is the checker
that the CUDA library is compared against, never a code path of the product;
``mockbird_b200`` does not import it and has no CPU fallback.

The arithmetic lives in ``oracle.c`` (a C restatement of the reference's WGSL
kernels, each function citing the reference file:line it follows); this module
only holds the numpy-side ring state and the ctypes plumbing.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

F32, BF16, F16 = 0, 1, 2
DTYPES = {"f32": F32, "bf16": BF16, "f16": F16}
HD = 64


class Geom(ctypes.Structure):
    _fields_ = [
        ("layers", ctypes.c_int32),
        ("streams", ctypes.c_int32),
        ("heads", ctypes.c_int32),
        ("capacity", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("wrap", ctypes.c_int32),
    ]


def build() -> None:
    """Compile oracle.c into liboracle.so (make; system gcc with OpenMP)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        P = ctypes.c_void_p
        i32 = ctypes.c_int32
        G = ctypes.POINTER(Geom)
        L.orc_rope_table.argtypes = [i32, ctypes.c_double, P]
        L.orc_rope_rows.argtypes = [i32, i32, P, i32, P, P, P, i32]
        L.orc_reset.argtypes = [G, P, i32]
        L.orc_rope_split_ring.argtypes = [G, P, P, P, i32, i32, P, P, P]
        L.orc_rope_split_ring.restype = ctypes.c_int
        L.orc_attend_ring.argtypes = [G, P, P, i32, i32, P, P, P, i32, P, i32]
        L.orc_append_attend.argtypes = [G, P, P, P, i32, i32, P, P, P, P, i32]
        L.orc_append_attend.restype = ctypes.c_int
        L.orc_gather.argtypes = [G, P, P, i32, i32, i32, P, P, P]
        L.orc_gather.restype = i32
        L.orc_prefill.argtypes = [G, P, P, P, i32, i32, P, i32, P, P, i32]
        L.orc_prefill.restype = ctypes.c_int
        L.orc_round_to.argtypes = [i32, P, P, ctypes.c_size_t]
        L.orc_xorshift_js.argtypes = [ctypes.POINTER(ctypes.c_uint32), ctypes.c_int64, P]
        L.orc_xorshift_js_f64.argtypes = [ctypes.POINTER(ctypes.c_uint32), ctypes.c_int64, P]
        _lib = L
    return _lib


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data_as(ctypes.c_void_p)


def rope_table(positions: int, theta: float = 10000.0) -> np.ndarray:
    """[positions][64] float32: (cos, sin) pairs per frequency, fp64 angles."""
    tab = np.empty((positions, HD), np.float32)
    lib().orc_rope_table(positions, theta, _p(tab))
    return tab


def rope_rows(x: np.ndarray, positions, tab: np.ndarray) -> np.ndarray:
    """RoPE of [rows][heads*64] rows at per-row positions (fp32, no FMA)."""
    x = np.ascontiguousarray(x, np.float32)
    rows, width = x.shape
    pos = np.ascontiguousarray(positions, np.int32)
    out = np.empty_like(x)
    lib().orc_rope_rows(rows, width // HD, _p(x), width, _p(pos), _p(tab), _p(out), width)
    return out


def round_to(dtype: str, x: np.ndarray) -> np.ndarray:
    """Round fp32 values to the storage dtype (nearest-even) and back."""
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty_like(x)
    lib().orc_round_to(DTYPES[dtype], _p(x), _p(out), x.size)
    return out


class Ring:
    """Host copy of the ring state: kv[layer][stream][2][head][slot][64] + slot_pos."""

    def __init__(self, layers=12, streams=1, heads=12, capacity=570, dtype="f32", wrap=True,
                 max_position=None, theta=10000.0):
        self.g = Geom(layers, streams, heads, capacity, DTYPES[dtype], int(bool(wrap)))
        self.dtype = dtype
        self.heads = heads
        self.capacity = capacity
        elems = layers * streams * 2 * heads * capacity * HD
        self.kv = np.zeros(elems, np.float32 if dtype == "f32" else np.uint16)
        self.slot_pos = np.full((layers, streams, capacity), -1, np.int32)
        self.tab = rope_table(max_position or max(capacity, 1) * 4, theta)

    def reset(self, stream: int = -1) -> None:
        lib().orc_reset(ctypes.byref(self.g), _p(self.slot_pos), stream)

    def _check_pos(self, positions):
        if len(positions) and int(np.max(positions)) >= self.tab.shape[0]:
            self.tab = rope_table(int(np.max(positions)) * 2 + 1)

    def rope_split(self, layer, streams, positions, qkv: np.ndarray) -> np.ndarray:
        """ROPE_SPLIT_RING/_CODEC; returns the row block with Q roped in place."""
        s = np.ascontiguousarray(streams, np.int32)
        p = np.ascontiguousarray(positions, np.int32)
        self._check_pos(p)
        q = np.array(qkv, np.float32, order="C", copy=True)
        rc = lib().orc_rope_split_ring(ctypes.byref(self.g), _p(self.kv), _p(self.slot_pos), _p(self.tab),
                                       layer, len(s), _p(s), _p(p), _p(q))
        if rc:
            raise ValueError("position does not fit the (non-wrapping) ring")
        return q

    def attend(self, layer, streams, positions, q_rows: np.ndarray, mode: int = 0) -> np.ndarray:
        """ATTEND_RING/_CODEC (mode 0, fp32 tile mirror) or ref-decode attend (mode 1, fp64)."""
        s = np.ascontiguousarray(streams, np.int32)
        p = np.ascontiguousarray(positions, np.int32)
        q = np.ascontiguousarray(q_rows, np.float32)
        ctx = np.zeros((len(s), self.heads * HD), np.float32)
        lib().orc_attend_ring(ctypes.byref(self.g), _p(self.kv), _p(self.slot_pos), layer, len(s), _p(s), _p(p),
                              _p(q), q.shape[1], _p(ctx), mode)
        return ctx

    def append_attend(self, layer, streams, positions, qkv: np.ndarray, mode: int = 0):
        """rope_split then attend (decode.ts:527-552); returns (ctx, roped qkv)."""
        q = self.rope_split(layer, streams, positions, qkv)
        return self.attend(layer, streams, positions, q, mode), q

    def gather(self, layer, stream, position):
        """Live window in position order: (k [H][W][64], v, slots [W])."""
        W = min(position + 1, self.capacity)
        dt = np.float32 if self.dtype == "f32" else np.uint16
        k = np.zeros((self.heads, W, HD), dt)
        v = np.zeros((self.heads, W, HD), dt)
        slots = np.zeros(W, np.int32)
        lib().orc_gather(ctypes.byref(self.g), _p(self.kv), _p(self.slot_pos), layer, stream, position,
                         _p(k), _p(v), _p(slots))
        return k, v, slots

    def prefill(self, layer, streams, qkv: np.ndarray, q_round: bool = False):
        """ROPE_SPLIT_CACHE + ATTENTION_*; qkv [n][rows][2304] -> (ctx [n][rows][768], roped qkv)."""
        s = np.ascontiguousarray(streams, np.int32)
        q = np.array(qkv, np.float32, order="C", copy=True)
        n, rows = q.shape[0], q.shape[1]
        self._check_pos(np.array([rows], np.int32))
        ctx = np.zeros((n, rows, self.heads * HD), np.float32)
        rc = lib().orc_prefill(ctypes.byref(self.g), _p(self.kv), _p(self.slot_pos), _p(self.tab), layer, n,
                               _p(s), rows, _p(q), _p(ctx), int(q_round))
        if rc:
            raise ValueError("prefill rows exceed the ring capacity")
        return ctx, q

    def kv_view(self):
        """kv as [layers][streams][2][heads][capacity][64]."""
        g = self.g
        return self.kv.reshape(g.layers, g.streams, 2, g.heads, g.capacity, HD)


def xorshift32_stream(seed: int = 0x2F6E2B1):
    """The PRNG of tests/gpu/kernels.test.mjs:22-30, evaluated as JavaScript does.

    Returns rnd(count) -> float32 draws; rnd(count, keep=False) only advances.
    """
    state = ctypes.c_uint32(seed & 0xFFFFFFFF)

    def rnd(count: int, keep: bool = True):
        if not keep:
            lib().orc_xorshift_js(ctypes.byref(state), count, None)
            return None
        out = np.empty(count, np.float32)
        lib().orc_xorshift_js(ctypes.byref(state), count, _p(out))
        return out

    return rnd


def xorshift32_stream_f64(seed: int = 0x2F6E2B1):
    """The same PRNG with its draws in fp64, before any Float32Array store:
    rnd(count) -> float64 draws.  kernels.test.mjs scales some draws in fp64 before
    storing them (`rnd() * 0.1`), so `(rnd(n) * 0.1).astype(np.float32)` is what
    its arrays hold."""
    state = ctypes.c_uint32(seed & 0xFFFFFFFF)

    def rnd(count: int):
        out = np.empty(count, np.float64)
        lib().orc_xorshift_js_f64(ctypes.byref(state), count, _p(out))
        return out

    return rnd


def layer_norm(x: np.ndarray, g: np.ndarray, b: np.ndarray, eps: float = 1e-5) -> np.ndarray:
    """LAYERNORM_1 (kernels-decode.ts:168-200) over the last axis: two passes (mean,
    then the mean of squared deviations), statistics in fp64 rounded to fp32,
    (x - mean) / sqrt(var + eps) * g + b in fp32."""
    mean = x.mean(-1, keepdims=True, dtype=np.float64).astype(np.float32)
    d = x - mean
    var = (d.astype(np.float64) ** 2).mean(-1, keepdims=True).astype(np.float32)
    return (d / np.sqrt(var + np.float32(eps)) * g + b).astype(np.float32)


def gemm_bf16(x: np.ndarray, W: np.ndarray, b: np.ndarray) -> np.ndarray:
    """GEMV (kernels-decode.ts:127-142), y = b + x W with W [K, N] row-major, at the
    rounding points of the CUDA path's bf16 GEMMs: x rounded to bf16, W given
    already in bf16, products and sums exact (fp64), the result rounded to fp32."""
    return (round_to("bf16", x).astype(np.float64) @ W.astype(np.float64) + b).astype(np.float32)


def decoder_step(ring: "Ring", weights: np.ndarray, ffn: int, streams, positions, hidden: np.ndarray) -> np.ndarray:
    """The global decode step of tools/onnx-probe/ref-decode.mjs:207-235 (decodeStep)
    for several streams, with the rounding points of a bf16 GEMM path: matrices and
    GEMM inputs rounded to bf16, everything else fp32.  LayerNorm eps 1e-5
    (kernels-decode.ts:168-200), GELU tanh (kernels-decode.ts:373-390), attention
    through the ring's fp32 mirror.  hidden [n][H*64] in (embedded rows), ln_f out."""
    h = ring.heads * HD
    w = np.asarray(weights, np.float32)
    off = [0]

    def take(count, shape=None, mat=False):
        a = w[off[0]:off[0] + count]
        off[0] += count
        a = round_to("bf16", a) if mat else a
        return a.reshape(shape) if shape else a

    ln, gemm = layer_norm, gemm_bf16

    x = np.array(hidden, np.float32, copy=True)
    for layer in range(ring.g.layers):
        ln1w, ln1b = take(h), take(h)
        wa, ba = take(h * 3 * h, (h, 3 * h), True), take(3 * h)
        wp, bp = take(h * h, (h, h), True), take(h)
        ln2w, ln2b = take(h), take(h)
        wi, bi = take(h * ffn, (h, ffn), True), take(ffn)
        wo, bo = take(ffn * h, (ffn, h), True), take(h)
        qkv = gemm(ln(x, ln1w, ln1b), wa, ba)
        ctx, _ = ring.append_attend(layer, streams, positions, qkv)
        x = x + gemm(ctx, wp, bp)
        a = gemm(ln(x, ln2w, ln2b), wi, bi)
        a = (0.5 * a * (1 + np.tanh(0.7978845608028654 * (a + 0.044715 * a * a * a)))).astype(np.float32)
        x = x + gemm(a, wo, bo)
    return ln(x, take(h), take(h))


# ---------------------------------------------------------------- local head

def argmax_penalty(logits: np.ndarray, seen_words: np.ndarray, penalty: float) -> int:
    """Greedy pick with the repetition penalty for one row of logits.

    ARGMAX_PENALTY (src/lib/tts/engine/kernels-decode.ts:428-485) and
    argmaxPenalty (tools/onnx-probe/ref-decode.mjs:273-284): a logit s whose id
    has its bit set in `seen_words` (bit j of word j/32) becomes s / penalty when
    s >= 0 and s * penalty when s < 0 (fp32 arithmetic); the scan starts from
    (-1e30, id 0) and keeps the first id of a strictly larger value, so ties go
    to the lowest id and NaNs never win."""
    s = np.array(logits, np.float32, copy=True)
    bits = ((np.asarray(seen_words, np.uint32)[np.arange(s.size) >> 5] >> (np.arange(s.size) & 31)) & 1) != 0
    p = np.float32(penalty)
    pos = bits & (s >= 0)
    neg = bits & (s < 0)
    s[pos] = s[pos] / p
    s[neg] = s[neg] * p
    best, idx = np.float32(-1e30), 0
    valid = ~np.isnan(s)
    if valid.any():
        m = s[valid].max()
        if m > best:
            idx = int(np.flatnonzero(s == m)[0])
    return idx


def local_weight_count(hidden: int, ffn: int, codes: int, channels: int) -> int:
    """Length of the local head's fp32 weight array (one layer + ln_f, wte_slot,
    the two text-head columns, channels-1 audio embeddings, channels audio heads)."""
    h, f = hidden, ffn
    layer = 2 * h + h * 3 * h + 3 * h + h * h + h + 2 * h + h * f + f + f * h + h + 2 * h
    return layer + h + 2 * h + (channels - 1) * codes * h + channels * h * codes


def local_frame(ring: "Ring", weights: np.ndarray, ffn: int, codes: int, channels: int, penalty: float,
                streams, hidden: np.ndarray, seen: np.ndarray, forced=None):
    """One frame of the local head for n streams (DecodeRunner.nextFrame,
    src/lib/tts/engine/decode.ts:788-939; CPU form ref-decode.mjs:236-283 and
    :380-410), with the rounding points of the CUDA path: the layer as in
    `decoder_step` (bf16 GEMMs), ln_f rounded to bf16 before the bf16 audio-head
    GEMM (no bias), the text-head decision in fp32 columns.

    `ring`: one layer, capacity >= channels + 1.  `seen` [ring streams][channels]
    [codes/32] uint32 is updated in place.  `forced` [n][channels]: tokens that
    drive the chain (embedding and seen bits) instead of this oracle's own picks,
    so that a kernel's picks can be followed step by step.
    Returns (tokens [n][channels] int32 -- this oracle's own picks, cont [n] int32,
    logits [n][channels][codes] fp32 before the penalty, decide [n][2] fp64 --
    the audio_end and assistant_slot dot products)."""
    h = ring.heads * HD
    w = np.asarray(weights, np.float32)
    nd = local_weight_count(h, ffn, codes, channels) - (h + 2 * h + (channels - 1) * codes * h
                                                        + channels * h * codes)
    off = nd
    wte_slot = w[off:off + h]
    off += h
    cols = w[off:off + 2 * h].reshape(2, h)
    off += 2 * h
    emb = w[off:off + (channels - 1) * codes * h].reshape(channels - 1, codes, h)
    off += (channels - 1) * codes * h
    heads = round_to("bf16", w[off:off + channels * h * codes]).reshape(channels, h, codes)
    streams = np.asarray(streams, np.int64)
    n = len(streams)
    tokens = np.zeros((n, channels), np.int32)
    used = np.zeros((n, channels), np.int32)
    cont = np.zeros(n, np.int32)
    logits = np.zeros((n, channels, codes), np.float32)
    decide = np.zeros((n, 2), np.float64)
    for step in range(channels + 1):
        if step == 0:
            x = np.array(hidden, np.float32, copy=True)
        elif step == 1:
            x = np.repeat(wte_slot[None, :], n, axis=0)
        else:
            x = emb[step - 2][used[:, step - 2]].copy()
        hs = decoder_step(ring, w[:nd], ffn, streams, [step] * n, x)
        if step == 0:
            decide = hs.astype(np.float64) @ cols.T.astype(np.float64)
            cont = (decide[:, 1] >= decide[:, 0]).astype(np.int32)
            continue
        ch = step - 1
        lg = (round_to("bf16", hs).astype(np.float64) @ heads[ch].astype(np.float64)).astype(np.float32)
        logits[:, ch] = lg
        for i in range(n):
            mask = seen[streams[i], ch]
            tokens[i, ch] = argmax_penalty(lg[i], mask, penalty)
            t = int(forced[i][ch]) if forced is not None else int(tokens[i, ch])
            used[i, ch] = t
            mask[t >> 5] |= np.uint32(1 << (t & 31))
    return tokens, cont, logits, decide
