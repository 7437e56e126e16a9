"""CPU tests of the ONNX weight reader (mockbird_b200.onnx_weights, the restated
openOnnx of src/lib/tts/engine/onnxWeights.ts:124) on a synthetic model in the
layout of the published decode graphs (tests/golden/make_onnx_fixture.py), with
the checks of the reference's own loader test (tests/gpu/loader.test.mjs) where
they apply at this size, and the assembly of the decoder and local-head weight
arrays (the order mb_decoder_create / mb_local_head_create take)."""
import os
import sys

import numpy as np
import pytest

from mockbird_b200.onnx_weights import decoder_weights, local_head_weights, open_model, open_onnx

sys.path.insert(0, os.path.join(os.path.dirname(__file__), "golden"))
import make_onnx_fixture as fx  # noqa: E402


@pytest.fixture(scope="module")
def model(tmp_path_factory):
    d = str(tmp_path_factory.mktemp("onnx"))
    expect = fx.write_fixture(d)
    return d, expect, open_model(os.path.join(d, "global.onnx"), os.path.join(d, "global.data")), \
        open_model(os.path.join(d, "local.onnx"), os.path.join(d, "local.data"))


def test_named_parameters_resolve_through_aliases(model):
    _, expect, g, _ = model
    names = (["core.model.transformer.wte.weight", "core.model.transformer.ln_f.weight",
              "core.model.transformer.ln_f.bias"]
             + [f"core.model.audio_embeddings.{k}.weight" for k in range(fx.NVQ)]
             + [f"core.model.transformer.h.{i}.{n}" for i in range(fx.LAYERS)
                for n in ("ln_1.weight", "ln_2.weight", "attn.c_attn.bias", "mlp.fc_out.bias")])
    assert all(g.has(n) for n in names)
    for n in names:
        assert np.array_equal(g.get(n).data, np.asarray(expect["global:" + n]).ravel()), n


def test_layer_norm_scales_alias_layer_zero(model):
    _, _, g, _ = model
    ln0 = g.get("core.model.transformer.h.0.ln_1.weight")
    ln1 = g.get("core.model.transformer.h.1.ln_1.weight")
    assert (ln0.data == 1).all() and (ln1.data == 1).all()
    assert np.shares_memory(ln0.data, ln1.data) and ln1.source == "alias" and ln0.source == "external"
    # an alias of an alias (two Identity hops)
    two = g.get("core.model.transformer.h.1.ln_2.weight")
    assert np.shares_memory(two.data, g.get("core.model.transformer.h.0.ln_2.weight").data)


def test_matrices_group_by_shape_in_sidecar_order(model):
    _, expect, g, _ = model
    h, f = fx.HIDDEN, fx.FFN
    shapes = [f"{h}x{3 * h}", f"{h}x{h}", f"{h}x{f}", f"{f}x{h}"]
    assert [len(g.by_shape(s)) for s in shapes] == [fx.LAYERS] * 4
    for j, s in enumerate(shapes):  # layer-major by offset although the names do not sort that way
        for i, m in enumerate(g.by_shape(s)):
            assert np.array_equal(m, expect["global:mats"][i][j].ravel()), (s, i)


def test_external_weights_are_views_of_the_sidecar(model):
    d, _, g, _ = model
    side = np.memmap(os.path.join(d, "global.data"), dtype=np.uint8, mode="r")
    t = open_onnx(open(os.path.join(d, "global.onnx"), "rb").read(), side).get("core.model.transformer.wte.weight")
    assert t.source == "external" and np.shares_memory(t.data, side)
    assert t.dims == [fx.VOCAB, fx.HIDDEN]
    # an external tensor at an offset that is not 4-byte aligned is copied out
    u = open_onnx(open(os.path.join(d, "global.onnx"), "rb").read(), side).get("unaligned_external")
    assert u.offset % 4 == 2 and not np.shares_memory(u.data, side)


def test_inline_constants_and_raw_initializers(model):
    _, expect, g, _ = model
    a, b = g.get("const_a"), g.get("const_b")
    assert a.source == "inline-constant" and a.dims == [2, 3]
    assert np.array_equal(a.data, expect["global:const_a"]) and np.array_equal(b.data, expect["global:const_b"])
    r = g.get("inline_raw")
    assert r.source == "inline-raw" and r.offset == -1 and np.array_equal(r.data, expect["global:inline_raw"])


def test_first_tensor_of_a_name_wins_and_only_fp32_is_read(model):
    _, expect, g, _ = model
    assert np.array_equal(g.get("core.model.transformer.ln_f.bias").data,
                          expect["global:core.model.transformer.ln_f.bias"])
    assert not g.has("int64_shape")
    with pytest.raises(KeyError, match="missing parameter nope"):
        g.get("nope")


def test_weight_inventory(model):
    _, _, g, _ = model
    h, f = fx.HIDDEN, fx.FFN
    per_layer = 4 * h * h + 2 * h * f + (3 * h + 3 * h + f + h)  # matrices + biases and LN biases
    scales = 2 * h  # layer 0's two LN scales (the other layers alias them)
    total_f32 = sum(g.get(n).data.size for n in g.names() if g.get(n).source != "alias")
    # + ln_f, the Constant (one tensor per output: 2 x 6), the inline raw (5), the unaligned external (7)
    want = (fx.LAYERS * per_layer + scales + fx.VOCAB * h + fx.NVQ * fx.CODES * h + 2 * h + 2 * 6 + 5 + 7)
    assert total_f32 == want


def test_decoder_weight_array(model):
    _, e, g, _ = model
    h, f = fx.HIDDEN, fx.FFN
    w = decoder_weights(g, layers=fx.LAYERS, hidden=h, ffn=f)
    parts = []
    for i in range(fx.LAYERS):
        p = f"global:core.model.transformer.h.{i}."
        m = e["global:mats"][i]
        parts += [e[p + "ln_1.weight"], e[p + "ln_1.bias"], m[0], e[p + "attn.c_attn.bias"], m[1],
                  e[p + "attn.c_proj.bias"], e[p + "ln_2.weight"], e[p + "ln_2.bias"], m[2], e[p + "mlp.fc_in.bias"],
                  m[3], e[p + "mlp.fc_out.bias"]]
    parts += [e["global:core.model.transformer.ln_f.weight"], e["global:core.model.transformer.ln_f.bias"]]
    assert np.array_equal(w, np.concatenate([np.ravel(x) for x in parts]))
    with pytest.raises(ValueError, match="expected 3"):
        decoder_weights(g, layers=3, hidden=h, ffn=f)


def test_local_head_weight_array(model):
    _, e, g, loc = model
    h, f, codes = fx.HIDDEN, fx.FFN, fx.CODES
    channels = 4
    w = local_head_weights(loc, g, fx.ASSISTANT_SLOT, fx.AUDIO_END, hidden=h, ffn=f, codes=codes, channels=channels)
    p = "local:model.local_transformer.h.0."
    m = e["local:mats"][0]
    parts = [e[p + "ln_1.weight"], e[p + "ln_1.bias"], m[0], e[p + "attn.c_attn.bias"], m[1], e[p + "attn.c_proj.bias"],
             e[p + "ln_2.weight"], e[p + "ln_2.bias"], m[2], e[p + "mlp.fc_in.bias"], m[3], e[p + "mlp.fc_out.bias"],
             e["local:model.local_transformer.ln_f.weight"], e["local:model.local_transformer.ln_f.bias"],
             e["global:core.model.transformer.wte.weight"][fx.ASSISTANT_SLOT],
             e["local:text_head"][:, fx.AUDIO_END], e["local:text_head"][:, fx.ASSISTANT_SLOT]]
    parts += [e[f"global:core.model.audio_embeddings.{k}.weight"] for k in range(channels - 1)]
    parts += e["local:heads"][:channels]
    assert np.array_equal(w, np.concatenate([np.ravel(x) for x in parts]))


def test_truncated_or_foreign_bytes_raise():
    with pytest.raises(ValueError):
        open_onnx(b"\x08", b"")  # a key with no value
    with pytest.raises(ValueError, match="no GraphProto"):
        open_onnx(b"\x08\x08", b"")  # ir_version only
    with pytest.raises(ValueError, match="wire type"):
        open_onnx(b"\x0b", b"")  # wire type 3 (group start)
