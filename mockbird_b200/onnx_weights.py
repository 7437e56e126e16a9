"""The ONNX weight reader of the reference engine, restated for this library's host side.

Mockbird does not run ONNX graphs: its engine reads the published MOSS-TTS-Nano
decode graphs only for their weights, through a small protobuf walker
(liyu1981/mockbird src/lib/tts/engine/onnxWeights.ts:124 `openOnnx`) and then
picks the per-layer tensors by name and by shape (prefill.ts:78
`resolveLayerWeights`, decodeWeights.ts `resolveLocalWeights`, gpu.ts:345-360).
This module does the same over numpy views, so the weights of a real model
directory can feed `mb_decoder_create` and `mb_local_head_create`
(include/mockbird_kv.h) in the order they take:

    open_onnx(onnx_bytes, sidecar)        WeightTable (get / has / names / size / by_shape)
    decoder_weights(table, ...)           the flat fp32 array of mb_decoder_create
    local_head_weights(local, global_, ...)   the flat fp32 array of mb_local_head_create

The reader follows openOnnx rule for rule:
  * initializers (GraphProto field 5) of element type 1 (fp32) only; one with an
    external-data entry "length" is a view of `length` bytes at `offset` of the
    sidecar (copied only when the offset is not 4-byte aligned), otherwise its
    inline raw_data (>= 4 bytes) is copied;
  * Constant nodes give their "value" tensor (fp32 raw_data) to every output;
  * Identity nodes with one input and one output are aliases, resolved through
    at most 8 hops (the LayerNorm scales of layers 1..11 alias layer 0's);
  * the first tensor of a name wins;
  * by_shape("KxN") lists the external tensors of those dims in sidecar order,
    which is the export's layer-major order (c_attn, c_proj, fc_in, fc_out): the
    anonymous onnx::MatMul_* names do not sort that way.
Protobuf wire types 0, 1, 2 and 5 are read; any other raises, as the reference does.
"""
from __future__ import annotations

import os
from dataclasses import dataclass

import numpy as np

# element sizes of the ONNX data types the reference knows (onnxWeights.ts:16)
ELEM_SIZE = {1: 4, 6: 4, 7: 8, 10: 2, 11: 8}


def _varint(buf, i: int) -> tuple[int, int]:
    result, shift = 0, 0
    while True:
        if i >= len(buf):
            raise ValueError("truncated protobuf varint")
        byte = buf[i]
        i += 1
        result += (byte & 0x7F) << shift
        if not byte & 0x80:
            return result, i
        shift += 7


def _fields(buf: memoryview):
    """Yield (field number, wire type, value) of a protobuf message: an int for
    wire type 0, a memoryview of the payload for wire types 1, 2 and 5."""
    i, n = 0, len(buf)
    while i < n:
        key, i = _varint(buf, i)
        field, wire = key >> 3, key & 7
        if wire == 0:
            v, i = _varint(buf, i)
            yield field, wire, v
        elif wire == 1:
            yield field, wire, buf[i:i + 8]
            i += 8
        elif wire == 2:
            ln, i = _varint(buf, i)
            yield field, wire, buf[i:i + ln]
            i += ln
        elif wire == 5:
            yield field, wire, buf[i:i + 4]
            i += 4
        else:
            raise ValueError(f"unsupported protobuf wire type {wire}")


def _text(b: memoryview) -> str:
    return bytes(b).decode("utf-8")


def _tensor_proto(buf: memoryview):
    """(name, dims, elem type, raw_data or None, external-data dict) of a TensorProto."""
    dims, external = [], {}
    name, elem, raw = "", 0, None
    for f, w, v in _fields(buf):
        if f == 1 and w == 0:
            dims.append(v)
        elif f == 2:
            elem = v
        elif f == 8:
            name = _text(v)
        elif f == 9:
            raw = v
        elif f == 13 and w == 2:
            key = value = ""
            for a, _, x in _fields(v):
                if a == 1:
                    key = _text(x)
                elif a == 2:
                    value = _text(x)
            external[key] = value
    return name, dims, elem, raw, external


def _float32(base: np.ndarray, byte_offset: int, byte_length: int, force_copy: bool) -> np.ndarray:
    """byte_length // 4 fp32 values at byte_offset of the uint8 array `base`: a
    view, or a copy when forced or when the offset is not 4-byte aligned."""
    count = byte_length // 4
    raw = base[byte_offset:byte_offset + count * 4]
    if len(raw) != count * 4:
        raise ValueError(f"tensor bytes [{byte_offset}, {byte_offset + count * 4}) lie outside the buffer")
    if force_copy or byte_offset % 4:
        return np.frombuffer(raw.tobytes(), dtype="<f4")
    return raw.view("<f4")


@dataclass
class Tensor:
    name: str
    dims: list
    data: np.ndarray      # fp32, flat
    source: str           # "external" | "inline-constant" | "inline-raw" | "alias"
    offset: int           # byte offset in the sidecar, -1 for inline tensors


class WeightTable:
    """Tensors by graph name, Identity aliases followed (the reference's WeightTable)."""

    def __init__(self, table: dict, aliases: dict):
        self._table, self._aliases = table, aliases

    def _resolve(self, name: str) -> str:
        current = name
        for _ in range(8):
            if current in self._table:
                return current
            nxt = self._aliases.get(current)
            if nxt is None:
                break
            current = nxt
        return current

    def get(self, name: str) -> Tensor:
        t = self._table.get(self._resolve(name))
        if t is None:
            raise KeyError(f"missing parameter {name}")
        return t

    def has(self, name: str) -> bool:
        return self._resolve(name) in self._table

    def names(self) -> list:
        return list(self._table)

    @property
    def size(self) -> int:
        return len(self._table)

    def by_shape(self, dims: str) -> list:
        """The data of the external tensors of dims "AxB", in sidecar order."""
        found = [t for t in self._table.values()
                 if t.source == "external" and "x".join(map(str, t.dims)) == dims and t.offset >= 0]
        return [t.data for t in sorted(found, key=lambda t: t.offset)]


def open_onnx(onnx_bytes, sidecar) -> WeightTable:
    """Parse a model (bytes of the .onnx file) whose external data live in
    `sidecar` (bytes, or a uint8 array such as a np.memmap of the .data file)."""
    model = memoryview(bytes(onnx_bytes)) if not isinstance(onnx_bytes, memoryview) else onnx_bytes
    side = sidecar if isinstance(sidecar, np.ndarray) else np.frombuffer(sidecar, dtype=np.uint8)
    graph = None
    for f, _, v in _fields(model):
        if f == 7:
            graph = v
    if graph is None:
        raise ValueError("no GraphProto in model")
    table: dict = {}
    aliases: dict = {}

    def add(t: Tensor):
        if t.name not in table:
            table[t.name] = t

    for f, _, gv in _fields(graph):
        if f == 5:  # initializer
            name, dims, elem, raw, external = _tensor_proto(gv)
            if not ELEM_SIZE.get(elem) or elem != 1:
                continue  # fp32 only
            if external.get("length"):
                offset = int(external.get("offset", 0) or 0)
                length = int(external["length"])
                add(Tensor(name, dims, _float32(side, offset, length, False), "external", offset))
            elif raw is not None and len(raw) >= 4:
                add(Tensor(name, dims, _float32(np.frombuffer(raw, dtype=np.uint8), 0, len(raw), True),
                           "inline-raw", -1))
        elif f == 1:  # node
            op, ins, outs, attrs = "", [], [], []
            for a, _, w in _fields(gv):
                if a == 1:
                    ins.append(_text(w))
                elif a == 2:
                    outs.append(_text(w))
                elif a == 4:
                    op = _text(w)
                elif a == 5:
                    attr_name, payload = "", None
                    for x, _, y in _fields(w):
                        if x == 1:
                            attr_name = _text(y)
                        elif x == 5:
                            payload = y
                    if payload is not None:
                        attrs.append((attr_name, payload))
            if op == "Identity" and len(ins) == 1 and len(outs) == 1:
                aliases[outs[0]] = ins[0]
            if op == "Constant":
                for attr_name, payload in attrs:
                    if attr_name != "value":
                        continue
                    _, dims, elem, raw, _ = _tensor_proto(payload)
                    if elem != 1 or raw is None or len(raw) < 4:
                        continue
                    data = _float32(np.frombuffer(raw, dtype=np.uint8), 0, len(raw), True)
                    for out in outs:
                        add(Tensor(out, dims, data, "inline-constant", -1))

    wt = WeightTable(table, aliases)
    for alias, target in aliases.items():  # the LayerNorm scales of layers 1..11
        if alias in table:
            continue
        t = table.get(wt._resolve(target))
        if t is not None:
            add(Tensor(alias, t.dims, t.data, "alias", t.offset))
    return wt


def open_model(onnx_path: str, data_path: str) -> WeightTable:
    """open_onnx over files; the sidecar is memory-mapped, so external tensors
    are views of the mapping (nothing is read until used)."""
    with open(onnx_path, "rb") as f:
        model = f.read()
    side = np.memmap(data_path, dtype=np.uint8, mode="r") if os.path.getsize(data_path) else np.zeros(0, np.uint8)
    return open_onnx(model, side)


# ---------------------------------------------------------------- the engine's weight sets

def _take(parts: list, t, count: int, what: str):
    a = np.asarray(t, dtype=np.float32).ravel()
    if a.size != count:
        raise ValueError(f"{what}: {a.size} values, expected {count}")
    parts.append(a)


def _layer_parts(table: WeightTable, prefix: str, i: int, mats, hidden: int, ffn: int, parts: list):
    h, f = hidden, ffn
    p = f"{prefix}.h.{i}."
    c_attn, c_proj, fc_in, fc_out = mats
    _take(parts, table.get(p + "ln_1.weight").data, h, p + "ln_1.weight")
    _take(parts, table.get(p + "ln_1.bias").data, h, p + "ln_1.bias")
    _take(parts, c_attn[i], h * 3 * h, f"c_attn of layer {i}")
    _take(parts, table.get(p + "attn.c_attn.bias").data, 3 * h, p + "attn.c_attn.bias")
    _take(parts, c_proj[i], h * h, f"c_proj of layer {i}")
    _take(parts, table.get(p + "attn.c_proj.bias").data, h, p + "attn.c_proj.bias")
    _take(parts, table.get(p + "ln_2.weight").data, h, p + "ln_2.weight")
    _take(parts, table.get(p + "ln_2.bias").data, h, p + "ln_2.bias")
    _take(parts, fc_in[i], h * f, f"fc_in of layer {i}")
    _take(parts, table.get(p + "mlp.fc_in.bias").data, f, p + "mlp.fc_in.bias")
    _take(parts, fc_out[i], f * h, f"fc_out of layer {i}")
    _take(parts, table.get(p + "mlp.fc_out.bias").data, h, p + "mlp.fc_out.bias")


def _matrices(table: WeightTable, hidden: int, ffn: int, layers: int, what: str):
    h, f = hidden, ffn
    mats = [table.by_shape(f"{h}x{3 * h}"), table.by_shape(f"{h}x{h}"), table.by_shape(f"{h}x{f}"),
            table.by_shape(f"{f}x{h}")]
    have = min(len(m) for m in mats)
    if have < layers:
        raise ValueError(f"{what}: {have} layers of [c_attn, c_proj, fc_in, fc_out] matrices, expected {layers}")
    return mats


def decoder_weights(table: WeightTable, layers: int = 12, hidden: int = 768, ffn: int = 3072,
                    prefix: str = "core.model.transformer") -> np.ndarray:
    """The global transformer's weights in mb_decoder_create's order (per layer
    ln_1, c_attn, c_proj, ln_2, fc_in, fc_out; then ln_f), picked as
    resolveLayerWeights (prefill.ts:78-108) picks them: matrices by shape in
    sidecar order, vectors by name."""
    mats = _matrices(table, hidden, ffn, layers, "global transformer")
    parts: list = []
    for i in range(layers):
        _layer_parts(table, prefix, i, mats, hidden, ffn, parts)
    _take(parts, table.get(prefix + ".ln_f.weight").data, hidden, prefix + ".ln_f.weight")
    _take(parts, table.get(prefix + ".ln_f.bias").data, hidden, prefix + ".ln_f.bias")
    return np.concatenate(parts)


def local_head_weights(local: WeightTable, global_: WeightTable, audio_assistant_slot_token_id: int,
                       audio_end_token_id: int, hidden: int = 768, ffn: int = 3072, codes: int = 1024,
                       channels: int = 16, vocab: int | None = None) -> np.ndarray:
    """The local head's weights in mb_local_head_create's order, picked as
    resolveLocalWeights (decodeWeights.ts) and the engine's embedding tables
    (gpu.ts:353-357) pick them: the local layer and ln_f
    (model.local_transformer.*), the wte row of audio_assistant_slot_token_id,
    the text-head columns audio_end_token_id and audio_assistant_slot_token_id,
    the audio embeddings 0..channels-2 (core.model.audio_embeddings.k) and the
    audio heads 0..channels-1 (the [hidden][codes] matrices in sidecar order)."""
    h = hidden
    mats = _matrices(local, hidden, ffn, 1, "local transformer")
    parts: list = []
    _layer_parts(local, "model.local_transformer", 0, mats, hidden, ffn, parts)
    _take(parts, local.get("model.local_transformer.ln_f.weight").data, h, "model.local_transformer.ln_f.weight")
    _take(parts, local.get("model.local_transformer.ln_f.bias").data, h, "model.local_transformer.ln_f.bias")
    wte = global_.get("core.model.transformer.wte.weight")
    if vocab is None:
        vocab = wte.data.size // h
    wte_rows = np.asarray(wte.data).reshape(vocab, h)
    _take(parts, wte_rows[audio_assistant_slot_token_id], h, "wte row of the assistant slot")
    text = local.by_shape(f"{h}x{vocab}")
    if not text:
        raise ValueError(f"local transformer: no {h}x{vocab} text head")
    text_head = np.asarray(text[0]).reshape(h, vocab)
    _take(parts, text_head[:, audio_end_token_id], h, "text head column audio_end")
    _take(parts, text_head[:, audio_assistant_slot_token_id], h, "text head column assistant_slot")
    for k in range(channels - 1):
        name = f"core.model.audio_embeddings.{k}.weight"
        _take(parts, global_.get(name).data, codes * h, name)
    heads = local.by_shape(f"{h}x{codes}")
    if len(heads) < channels:
        raise ValueError(f"local transformer: {len(heads)} audio heads of {h}x{codes}, expected {channels}")
    for k in range(channels):
        _take(parts, heads[k], h * codes, f"audio head {k}")
    return np.concatenate(parts)
