"""Generates the golden fixtures in tests/golden/ from the REFERENCE ITSELF.

Every expected output here is produced by pure-c-llm's own attention code,
compiled from its unmodified sources into oracle/_ref/ by oracle/Makefile:
  - train.c attention_forward / attention_backward (train.c:339-407)
  - transformer.c cached_attention (transformer.c:203-248)
  - train.c matmul_forward (train.c:181-211), as the Q, K, V projections
Inputs come from the seeded splitmix64/Box-Muller generator (synth.py) and
are stored in the fixture next to the outputs, so the fixtures do not depend
on the generator staying bit-identical.  The INT8 fixture's codes/scales come
from the reference's own quantize_A (gemm_bench.c:225-236) applied per (token,
head) slice (oracle/ref_quant_harness.c), and its expected output
from the reference's cached_attention over the dequantised cache.

Run from the repository root:  python tests/golden/make_golden.py
(needs the reference tree to build oracle/_ref; the fixtures are committed).
"""
import os
import sys

import numpy as np

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), "..", ".."))
sys.path.insert(0, os.path.join(ROOT, "pure-c-llm_b200"))
sys.path.insert(0, ROOT)
import synth  # noqa: E402
from oracle import oracle as O  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))


def save(name, **arrays):
    np.savez_compressed(os.path.join(OUT, name + ".npz"), **arrays)
    print(name, {k: v.shape for k, v in arrays.items()})


def fwd_case(name, seed, B, T, H, d):
    q = synth.normal(seed, (B * T, H * d), 0.0, 0.5)
    k = synth.normal(seed + 1, (B * T, H * d), 0.0, 0.5)
    v = synth.normal(seed + 2, (B * T, H * d), 0.0, 0.5)
    att, probs = O.ref_attention_forward(q, k, v, B, T, H, d)
    save(name, q=q, k=k, v=v, att=att, probs=probs, shape=np.array([B, T, H, d]))


def bwd_case(name, seed, B, T, H, d):
    q = synth.normal(seed, (B * T, H * d), 0.0, 0.5)
    k = synth.normal(seed + 1, (B * T, H * d), 0.0, 0.5)
    v = synth.normal(seed + 2, (B * T, H * d), 0.0, 0.5)
    do = synth.normal(seed + 3, (B * T, H * d), 0.0, 1.0)
    att, probs = O.ref_attention_forward(q, k, v, B, T, H, d)
    dq, dk, dv = O.ref_attention_backward(do, q, k, v, probs, B, T, H, d)
    save(name, q=q, k=k, v=v, do=do, att=att, dq=dq, dk=dk, dv=dv, shape=np.array([B, T, H, d]))


def decode_case(name, seed, H, d, t_max, positions):
    rows = max(positions) + 1
    kc = np.zeros((t_max, H * d), np.float32)
    vc = np.zeros((t_max, H * d), np.float32)
    kc[:rows] = synth.normal(seed, (rows, H * d))
    vc[:rows] = synth.normal(seed + 1, (rows, H * d))
    q = synth.normal(seed + 2, (len(positions), H * d))
    outs = np.stack([O.ref_cached_attention(q[i], kc, vc, p, H, d, t_max) for i, p in enumerate(positions)])
    save(name, q=q, kcache=kc[:rows], vcache=vc[:rows], out=outs, positions=np.array(positions),
         shape=np.array([H, d, t_max]))


def quant_case(name, seed, rows, H, d):
    x = synth.normal(seed, (rows, H * d), 0.0, 1.0)
    x[0, :d] = 0.0                                   # all-zero head: amax floor 1e-8
    x[1, :d] = 0.0
    x[1, 0] = 127.0                                  # scale exactly 1: ties at .5 below
    x[1, 1:9] = [2.5, -2.5, 0.5, -0.5, 1.5, -1.5, 126.5, -126.5]
    x[2, :d] = np.linspace(-3.0, 3.0, d)
    x[3, d:2 * d] = 1e-9                             # below the floor
    x[4, :d] *= 1e4                                  # large magnitudes
    codes, scales = O.ref_quantize_kv_int8(x, H, d)
    save(name, x=x, codes=codes, scales=scales, shape=np.array([H, d]))


def int8_decode_case(name, seed, H, d, t_max, pos):
    rows = pos + 1
    kc = synth.normal(seed, (rows, H * d))
    vc = synth.normal(seed + 1, (rows, H * d))
    q = synth.normal(seed + 2, (H * d,))
    kq, ks = O.ref_quantize_kv_int8(kc, H, d)
    vq, vs = O.ref_quantize_kv_int8(vc, H, d)
    kd = np.zeros((t_max, H * d), np.float32)
    vd = np.zeros((t_max, H * d), np.float32)
    kd[:rows] = O.dequantize_kv_int8(kq, ks, H, d)
    vd[:rows] = O.dequantize_kv_int8(vq, vs, H, d)
    out = O.ref_cached_attention(q, kd, vd, pos, H, d, t_max)
    save(name, q=q, kcodes=kq, kscale=ks, vcodes=vq, vscale=vs, out=out, pos=np.array(pos),
         shape=np.array([H, d, t_max]))


def qkv_case(name, seed, M, K, N):
    """Q, K, V projections of train.c:517-519 through the reference's own
    matmul_forward (train.c:181-211; its AVX-512 micro-kernel when M % 8 == 0
    and N % 16 == 0, else its i-k-j loop)."""
    x = synth.normal(seed, (M, K))
    ws = [synth.normal(seed + 1 + i, (K, N), 0, 0.02) for i in range(3)]
    bs = [synth.normal(seed + 4 + i, (N,), 0, 0.1) for i in range(3)]
    outs = [O.ref_matmul_forward(x, w, b) for w, b in zip(ws, bs)]
    save(name, x=x, wq=ws[0], wk=ws[1], wv=ws[2], bq=bs[0], bk=bs[1], bv=bs[2], q=outs[0], k=outs[1],
         v=outs[2], shape=np.array([M, K, N]))


if __name__ == "__main__":
    fwd_case("fwd_h4_d32", 101, B=2, T=37, H=4, d=32)
    fwd_case("fwd_h2_d64", 111, B=1, T=65, H=2, d=64)
    fwd_case("fwd_h2_d128", 121, B=1, T=9, H=2, d=128)
    fwd_case("fwd_h2_d96", 131, B=1, T=17, H=2, d=96)
    fwd_case("fwd_t1", 141, B=1, T=1, H=2, d=64)
    bwd_case("bwd_h2_d64", 201, B=1, T=65, H=2, d=64)
    bwd_case("bwd_h4_d32", 211, B=2, T=33, H=4, d=32)
    decode_case("decode_h4_d32", 301, H=4, d=32, t_max=512, positions=[0, 63, 150])
    decode_case("decode_h2_d64", 311, H=2, d=64, t_max=512, positions=[0, 40, 511 - 470])
    quant_case("quant_h4_d32", 401, rows=20, H=4, d=32)
    int8_decode_case("int8_decode_h2_d64", 501, H=2, d=64, t_max=512, pos=90)
    qkv_case("qkv_m72_k96_n64", 601, M=72, K=96, N=64)
    qkv_case("qkv_m37_k52_n36", 611, M=37, K=52, N=36)
