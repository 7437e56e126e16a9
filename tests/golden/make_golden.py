"""Generate the golden fixtures under tests/golden/ (run once, in a container that
has the reference tree; the fixtures are committed so nothing reads the reference
at test time).

    python tests/golden/make_golden.py --reference <path of the reference tree>

Outputs
-------
layer0_kv.npz
    From the reference's ONNX-Runtime goldens
    (tests/fixtures/golden/prefill-{8,195}rows-*.{u32,f32}, captured from
    moss_tts_prefill.onnx under onnxruntime-node 1.30.0, per
    tests/fixtures/golden/prefill-reference.json):
      ids      [195, 17] u32   prompt rows (the 8-row case is their prefix)
      rows     [R]       i32   which rows of the 195-row case are stored
      k, v     [R, 12, 64] f32 layer-0 post-RoPE key / raw value cache rows
      k8_equal              the 8-row K/V files equal the first 8 rows of the
                            195-row files (checked here, byte for byte)
    Rows with identical ids have identical pre-RoPE K and identical V at layer
    0 (MOSS-TTS-Nano has no absolute position embedding), so every pair of such
    rows pins the RoPE convention: K[j] = RoPE_j(RoPE_i^-1(K[i])).

kat_attention_n512.npz
    The known answer of tests/gpu/kernels.test.mjs test 4 ("attention vs ring
    cache N=512 heads=12", :272-377): inputs are the test's own xorshift32
    stream (seed 0x2f6e2b1) after the draws of tests 1-3 (1 774 144 values),
    k[i] / v[i] drawn interleaved, then q; the expected output is the test's
    float64 JavaScript reference restated below in numpy (not by the oracle).
      out      [768] f32   expected context
      skip     int         draws consumed before test 4
      k_sum, v_sum, q_sum  float64 sums of the inputs (regeneration check)

kat_argmax_c1024.npz
    The known answer of kernels.test.mjs test 5 ("argmax over 1024 logits (tie ->
    lowest id)", :379-436): 1024 logits drawn from the same stream right after
    test 4's inputs; the expected id is the test's own JavaScript scan (first id
    of a strictly larger value), restated below in plain Python.
      best     int         expected id
      skip     int         draws consumed before test 5
      logits_sum           float64 sum of the logits (regeneration check)

kat_layernorm_d768.npz
    The known answer of kernels.test.mjs test 1 ("layernorm d=768 eps=1e-5",
    :90-163), the first draws of the stream; the expected row is the test's
    float64 loop restated below in plain Python.
      out      [768] f32   expected row
      x_sum, b_sum         float64 sums of the inputs (regeneration check)

kat_gemv_k768_n2304.npz
    The known answer of kernels.test.mjs test 2 ("gemv [K=768, N=2304] c_attn",
    :165-223), drawn right after test 1's inputs; the expected vector is the
    test's float64 loop, summed in its order.
      out      [2304] f32  expected y = bias + x W
      skip     int         draws consumed before test 2
      x_sum, w_sum, bias_sum  float64 sums of the inputs (regeneration check)
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import oracle  # noqa: E402  (the JS-exact PRNG lives in the oracle's C code)

H, HD, D = 12, 64, 768
# draws of kernels.test.mjs before test 4: layernorm 2*768, gemv 768 + 768*2304 + 2304, rope 64
SKIP_BEFORE_TEST4 = 2 * D + (D + D * 3 * D + 3 * D) + HD
N_KAT = 512


def kat_inputs():
    rnd = oracle.xorshift32_stream(0x2F6E2B1)
    rnd(SKIP_BEFORE_TEST4, keep=False)
    kv = rnd(2 * N_KAT * H * HD)
    k = kv[0::2].copy()          # k[i] = rnd(); v[i] = rnd();  interleaved
    v = kv[1::2].copy()
    q = rnd(H * HD)
    return k, v, q


def kat_expected(k, v, q):
    """kernels.test.mjs:285-307 in float64: layout kv[(pos*H + h)*HD + d]."""
    kk = k.astype(np.float64).reshape(N_KAT, H, HD)
    vv = v.astype(np.float64).reshape(N_KAT, H, HD)
    qq = q.astype(np.float64).reshape(H, HD)
    scale = 1.0 / np.sqrt(HD)
    out = np.zeros((H, HD))
    for h in range(H):
        s = np.array([sum(float(qq[h, d]) * float(kk[j, h, d]) for d in range(HD)) for j in range(N_KAT)]) * scale
        e = np.exp(s - s.max())
        p = e / e.sum()
        for d in range(HD):
            acc = 0.0
            for j in range(N_KAT):
                acc += p[j] * vv[j, h, d]
            out[h, d] = acc
    return out.reshape(-1).astype(np.float32)


def kat_argmax():
    """kernels.test.mjs:381-386: logits[i] = rnd(); best = first id of the max."""
    skip = SKIP_BEFORE_TEST4 + 2 * N_KAT * H * HD + H * HD
    rnd = oracle.xorshift32_stream(0x2F6E2B1)
    rnd(skip, keep=False)
    logits = rnd(1024)
    best = 0
    for i in range(1, 1024):
        if logits[i] > logits[best]:
            best = i
    return logits, best, skip


def kat_layernorm():
    """kernels.test.mjs:90-109 (test 1, "layernorm d=768 eps=1e-5"): per i, x[i] =
    rnd()*4 then b[i] = rnd()*0.1 (scaled in fp64, stored fp32), g = 1; the
    expected row is the test's fp64 loop restated (sequential sums)."""
    rnd = oracle.xorshift32_stream_f64(0x2F6E2B1)
    d = rnd(2 * D)
    x = (d[0::2] * 4).astype(np.float32)
    b = (d[1::2] * 0.1).astype(np.float32)
    mean = 0.0
    for v in x:
        mean += float(v)
    mean /= D
    var = 0.0
    for v in x:
        var += (float(v) - mean) ** 2
    var /= D
    inv = 1.0 / np.sqrt(var + 1e-5)
    out = np.array([(float(x[i]) - mean) * inv * 1.0 + float(b[i]) for i in range(D)]).astype(np.float32)
    return x, b, out


def kat_gemv():
    """kernels.test.mjs:165-223 (test 2, "gemv [K=768, N=2304] c_attn"), drawn after
    test 1's 2*768 values: x[k] = rnd(), W[k*N+n] = rnd()*0.05, bias[n] = rnd()*0.02;
    the expected y[n] = bias[n] + sum_k x[k] W[k, n] is the test's fp64 loop, summed
    in its order (k ascending from the bias)."""
    K, N = D, 3 * D
    rnd = oracle.xorshift32_stream_f64(0x2F6E2B1)
    rnd(2 * D)
    x = rnd(K).astype(np.float32)
    W = (rnd(K * N) * 0.05).astype(np.float32).reshape(K, N)
    bias = (rnd(N) * 0.02).astype(np.float32)
    acc = bias.astype(np.float64)
    for k in range(K):
        acc = acc + float(x[k]) * W[k].astype(np.float64)
    return x, W, bias, acc.astype(np.float32)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="root of the reference tree")
    a = ap.parse_args()
    g = os.path.join(a.reference, "tests", "fixtures", "golden")

    ids = np.fromfile(os.path.join(g, "prefill-195rows-ids.u32"), np.uint32).reshape(195, 17)
    ids8 = np.fromfile(os.path.join(g, "prefill-8rows-ids.u32"), np.uint32).reshape(8, 17)
    K = np.fromfile(os.path.join(g, "prefill-195rows-layer0-k.f32"), np.float32).reshape(195, H, HD)
    V = np.fromfile(os.path.join(g, "prefill-195rows-layer0-v.f32"), np.float32).reshape(195, H, HD)
    K8 = np.fromfile(os.path.join(g, "prefill-8rows-layer0-k.f32"), np.float32).reshape(8, H, HD)
    V8 = np.fromfile(os.path.join(g, "prefill-8rows-layer0-v.f32"), np.float32).reshape(8, H, HD)
    k8_equal = bool((ids8 == ids[:8]).all() and (K8 == K[:8]).all() and (V8 == V[:8]).all())
    rows = np.array(list(range(0, 8)) + list(range(128, 195)), np.int32)
    np.savez_compressed(os.path.join(HERE, "layer0_kv.npz"), ids=ids, rows=rows, k=K[rows], v=V[rows],
                        k8_equal=np.array(k8_equal))

    k, v, q = kat_inputs()
    out = kat_expected(k, v, q)
    np.savez_compressed(os.path.join(HERE, "kat_attention_n512.npz"), out=out, skip=np.array(SKIP_BEFORE_TEST4),
                        k_sum=np.array(k.astype(np.float64).sum()), v_sum=np.array(v.astype(np.float64).sum()),
                        q_sum=np.array(q.astype(np.float64).sum()))
    logits, best, skip = kat_argmax()
    np.savez_compressed(os.path.join(HERE, "kat_argmax_c1024.npz"), best=np.array(best), skip=np.array(skip),
                        logits_sum=np.array(logits.astype(np.float64).sum()))
    x, b, out = kat_layernorm()
    np.savez_compressed(os.path.join(HERE, "kat_layernorm_d768.npz"), out=out,
                        x_sum=np.array(x.astype(np.float64).sum()), b_sum=np.array(b.astype(np.float64).sum()))
    x, W, bias, y = kat_gemv()
    np.savez_compressed(os.path.join(HERE, "kat_gemv_k768_n2304.npz"), out=y, skip=np.array(2 * D),
                        x_sum=np.array(x.astype(np.float64).sum()), w_sum=np.array(W.astype(np.float64).sum()),
                        bias_sum=np.array(bias.astype(np.float64).sum()))
    print("wrote kat_layernorm_d768.npz and kat_gemv_k768_n2304.npz")
    print("wrote layer0_kv.npz (rows %d, k8_equal=%s), kat_attention_n512.npz and kat_argmax_c1024.npz (best %d)"
          % (len(rows), k8_equal, best))


if __name__ == "__main__":
    main()
