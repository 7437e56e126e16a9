"""Write a small synthetic model in the layout of the published MOSS-TTS-Nano
decode graphs, for the tests of mockbird_b200.onnx_weights.

    python tests/golden/make_onnx_fixture.py OUT_DIR

The real graphs (moss_tts_decode_step.onnx + moss_tts_global_shared.data,
moss_tts_local_cached_step.onnx + moss_tts_local_shared.data) hold 715 MB of
weights that this image does not have.  This script writes two model/sidecar
pairs with the same structure at a small size (hidden 64, FFN 256, 2 global
layers, vocab 320, 16 codebooks of 128 codes), using its own protobuf encoder
(no onnx package): the weight sources the reader must handle are all present --
  * anonymous onnx::MatMul_<n> initializers in the sidecar, layer-major, named
    so that their names do not sort in layer order;
  * named vectors and embeddings in the sidecar;
  * the LayerNorm scales of layer 0 as initializers and those of the other
    layers as Identity aliases of them (two hops for one of them);
  * a Constant node with an inline fp32 value given to two outputs;
  * an inline raw_data initializer (copied out of the protobuf bytes);
  * an external tensor at an offset that is not 4-byte aligned;
  * an int64 initializer (skipped: fp32 only) and a duplicate name (first wins).
Returns (write_fixture) the expected tensors so the tests can compare.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HIDDEN, FFN, LAYERS, VOCAB, CODES, NVQ = 64, 256, 2, 320, 128, 16
ASSISTANT_SLOT, AUDIO_END = 9, 7


def _varint(n: int) -> bytes:
    out = bytearray()
    while True:
        b = n & 0x7F
        n >>= 7
        if n:
            out.append(b | 0x80)
        else:
            out.append(b)
            return bytes(out)


def _key(field: int, wire: int) -> bytes:
    return _varint(field << 3 | wire)


def _vint(field: int, n: int) -> bytes:
    return _key(field, 0) + _varint(n)


def _ld(field: int, payload: bytes) -> bytes:
    return _key(field, 2) + _varint(len(payload)) + payload


def _s(field: int, text: str) -> bytes:
    return _ld(field, text.encode())


def tensor_proto(name: str, dims, data_type: int = 1, raw: bytes | None = None, external=None) -> bytes:
    """TensorProto: dims (1, one varint each), data_type (2), name (8), raw_data (9),
    external_data (13: key 1, value 2), data_location (14, 1 = EXTERNAL)."""
    out = b"".join(_vint(1, d) for d in dims) + _vint(2, data_type) + _s(8, name)
    if raw is not None:
        out += _ld(9, raw)
    if external:
        for k, v in external:
            out += _ld(13, _s(1, k) + _s(2, v))
        out += _vint(14, 1)
    return out


def node(op: str, inputs, outputs, name: str = "", value: bytes | None = None) -> bytes:
    """NodeProto: input (1), output (2), name (3), op_type (4), attribute (5:
    name 1, t 5, type 20 = TENSOR)."""
    out = b"".join(_s(1, i) for i in inputs) + b"".join(_s(2, o) for o in outputs)
    if name:
        out += _s(3, name)
    out += _s(4, op)
    if value is not None:
        out += _ld(5, _s(1, "value") + _ld(5, value) + _vint(20, 4))
    return out


def model(nodes, initializers) -> bytes:
    """ModelProto: ir_version (1), graph (7: node 1, name 2, initializer 5)."""
    graph = b"".join(_ld(1, n) for n in nodes) + _s(2, "main") + b"".join(_ld(5, t) for t in initializers)
    return _vint(1, 8) + _ld(7, graph)


class _Sidecar:
    def __init__(self):
        self.buf = bytearray()

    def put(self, a: np.ndarray, pad_to: int = 64) -> tuple[int, int]:
        while len(self.buf) % pad_to:
            self.buf.append(0)
        off = len(self.buf)
        raw = np.ascontiguousarray(a, dtype="<f4").tobytes()
        self.buf += raw
        return off, len(raw)

    def put_unaligned(self, a: np.ndarray) -> tuple[int, int]:
        while len(self.buf) % 4 != 2:
            self.buf.append(0)
        off = len(self.buf)
        raw = np.ascontiguousarray(a, dtype="<f4").tobytes()
        self.buf += raw
        return off, len(raw)


def _ext(name, dims, loc):
    off, ln = loc
    return tensor_proto(name, dims, external=[("location", "shared.data"), ("offset", str(off)),
                                              ("length", str(ln))])


def _layer_mats(rng, h, f):
    return [rng.standard_normal((h, 3 * h)).astype(np.float32) * 0.05,
            rng.standard_normal((h, h)).astype(np.float32) * 0.05,
            rng.standard_normal((h, f)).astype(np.float32) * 0.05,
            rng.standard_normal((f, h)).astype(np.float32) * 0.05]


def _layer_vecs(rng, h, f):
    return {"attn.c_attn.bias": rng.standard_normal(3 * h).astype(np.float32) * 0.1,
            "attn.c_proj.bias": rng.standard_normal(h).astype(np.float32) * 0.1,
            "ln_1.bias": rng.standard_normal(h).astype(np.float32) * 0.1,
            "ln_2.bias": rng.standard_normal(h).astype(np.float32) * 0.1,
            "mlp.fc_in.bias": rng.standard_normal(f).astype(np.float32) * 0.1,
            "mlp.fc_out.bias": rng.standard_normal(h).astype(np.float32) * 0.1}


def write_fixture(out_dir: str, seed: int = 0) -> dict:
    """Write global.onnx/global.data and local.onnx/local.data into out_dir;
    return the tensors they hold, by name ("global:<name>", "local:<name>"), plus
    the matrices in layer order ("global:mats", "local:mats", "local:heads")."""
    os.makedirs(out_dir, exist_ok=True)
    rng = np.random.default_rng(seed)
    h, f = HIDDEN, FFN
    expect: dict = {}

    # ---------------- global: 2 layers, wte, 16 audio embeddings, ln_f
    side, inits, nodes = _Sidecar(), [], []
    ones = np.ones(h, np.float32)
    mats = []
    mat_no = [31, 107, 9, 12, 58, 4, 300, 77]  # onnx::MatMul_<n>: not in layer order by name
    for i in range(LAYERS):
        p = f"core.model.transformer.h.{i}."
        ms = _layer_mats(rng, h, f)
        mats.append(ms)
        for j, m in enumerate(ms):
            inits.append(_ext(f"onnx::MatMul_{mat_no[4 * i + j]}", m.shape, side.put(m)))
        for k, v in _layer_vecs(rng, h, f).items():
            inits.append(_ext(p + k, v.shape, side.put(v)))
            expect["global:" + p + k] = v
        ln_w2 = (1.0 + 0.01 * rng.standard_normal(h)).astype(np.float32)
        if i == 0:  # layer 0's scales are initializers; the other layers alias them
            inits.append(_ext(p + "ln_1.weight", (h,), side.put(ones)))
            inits.append(_ext(p + "ln_2.weight", (h,), side.put(ln_w2)))
            expect["global:" + p + "ln_1.weight"] = ones
            expect["global:" + p + "ln_2.weight"] = ln_w2
        else:
            q = "core.model.transformer.h.0."
            nodes.append(node("Identity", [q + "ln_1.weight"], [p + "ln_1.weight"]))
            nodes.append(node("Identity", ["alias_hop"], [p + "ln_2.weight"]))  # two hops
            nodes.append(node("Identity", [q + "ln_2.weight"], ["alias_hop"]))
            expect["global:" + p + "ln_1.weight"] = ones
            expect["global:" + p + "ln_2.weight"] = expect["global:" + q + "ln_2.weight"]
    expect["global:mats"] = mats
    wte = rng.standard_normal((VOCAB, h)).astype(np.float32)
    inits.append(_ext("core.model.transformer.wte.weight", wte.shape, side.put(wte)))
    expect["global:core.model.transformer.wte.weight"] = wte
    for k in range(NVQ):
        e = rng.standard_normal((CODES, h)).astype(np.float32)
        inits.append(_ext(f"core.model.audio_embeddings.{k}.weight", e.shape, side.put(e)))
        expect[f"global:core.model.audio_embeddings.{k}.weight"] = e
    lnf_w = (1.0 + 0.01 * rng.standard_normal(h)).astype(np.float32)
    lnf_b = (0.1 * rng.standard_normal(h)).astype(np.float32)
    inits.append(_ext("core.model.transformer.ln_f.weight", (h,), side.put(lnf_w)))
    inits.append(_ext("core.model.transformer.ln_f.bias", (h,), side.put(lnf_b)))
    expect["global:core.model.transformer.ln_f.weight"] = lnf_w
    expect["global:core.model.transformer.ln_f.bias"] = lnf_b
    # the other sources
    c = rng.standard_normal(6).astype(np.float32)
    nodes.insert(0, node("Constant", [], ["const_a", "const_b"], value=tensor_proto("", (2, 3), raw=c.tobytes())))
    expect["global:const_a"] = expect["global:const_b"] = c
    r = rng.standard_normal(5).astype(np.float32)
    inits.append(tensor_proto("inline_raw", (5,), raw=r.tobytes()))
    expect["global:inline_raw"] = r
    u = rng.standard_normal(7).astype(np.float32)
    inits.append(_ext("unaligned_external", (7,), side.put_unaligned(u)))
    expect["global:unaligned_external"] = u
    inits.append(tensor_proto("int64_shape", (3,), data_type=7, raw=np.arange(3, dtype="<i8").tobytes()))
    inits.append(_ext("core.model.transformer.ln_f.bias", (h,), side.put(lnf_b + 5.0)))  # duplicate: ignored
    with open(os.path.join(out_dir, "global.onnx"), "wb") as fh:
        fh.write(model(nodes, inits))
    with open(os.path.join(out_dir, "global.data"), "wb") as fh:
        fh.write(bytes(side.buf))

    # ---------------- local: one layer, ln_f, the text head, 16 audio heads
    side, inits, nodes = _Sidecar(), [], []
    p = "model.local_transformer.h.0."
    ms = _layer_mats(rng, h, f)
    expect["local:mats"] = [ms]
    for j, m in enumerate(ms):
        inits.append(_ext(f"onnx::MatMul_{900 - j}", m.shape, side.put(m)))
    for k, v in _layer_vecs(rng, h, f).items():
        inits.append(_ext(p + k, v.shape, side.put(v)))
        expect["local:" + p + k] = v
    for k in ("ln_1.weight", "ln_2.weight"):
        v = (1.0 + 0.01 * rng.standard_normal(h)).astype(np.float32)
        inits.append(_ext(p + k, (h,), side.put(v)))
        expect["local:" + p + k] = v
    for k in ("weight", "bias"):
        v = (1.0 + 0.01 * rng.standard_normal(h)).astype(np.float32) if k == "weight" else \
            (0.1 * rng.standard_normal(h)).astype(np.float32)
        inits.append(_ext("model.local_transformer.ln_f." + k, (h,), side.put(v)))
        expect["local:model.local_transformer.ln_f." + k] = v
    text = (rng.standard_normal((h, VOCAB)) / np.sqrt(h)).astype(np.float32)
    inits.append(_ext("onnx::MatMul_5", text.shape, side.put(text)))
    expect["local:text_head"] = text
    heads = []
    for k in range(NVQ):
        m = (rng.standard_normal((h, CODES)) * 0.1).astype(np.float32)
        heads.append(m)
        inits.append(_ext(f"onnx::MatMul_{1000 - k}", m.shape, side.put(m)))
    expect["local:heads"] = heads
    with open(os.path.join(out_dir, "local.onnx"), "wb") as fh:
        fh.write(model(nodes, inits))
    with open(os.path.join(out_dir, "local.data"), "wb") as fh:
        fh.write(bytes(side.buf))
    return expect


if __name__ == "__main__":
    write_fixture(sys.argv[1] if len(sys.argv) > 1 else "onnx_fixture")
