"""The edits a maintainer makes to the reference's own sources to route their
attention to libattn_b200, as text transformations.  The build recipe
(tests/integration/Makefile) and tests/test_link.py apply them to copies in a
temporary directory; nothing edited is kept in the repository.

  guard_gpu_kernels  gpu_kernels.cu: the attention section (lines 253-489:
                     k_causal_softmax, k_softmax_bwd, the hand GEMMs, attn_fwd,
                     attn_bwd) inside #ifndef ATTN_EXTERNAL, so a build with
                     -DATTN_EXTERNAL takes attn_fwd / attn_bwd from the library.
  shrink_trainer     train_kaggle.cu: a_probs and s_Dbuf shrunk from B*H*T*T
                     floats to B*H*T and 2*B*H*T, with the library in its
                     lse-only probs mode.
  fuse_qkv           train_kaggle.cu (on top of shrink_trainer): the three
                     gemm_nn calls of the Q, K and V projections
                     (train_kaggle.cu:152-154) replaced by one attn_qkv_proj.
  route_generate     generate.c: the per-head attention loop of block()
                     (generate.c:129-152) replaced by one call of
                     attn_cached_attention_host_ex.

Usage: python ref_edits.py <reference dir> <out dir>  (writes
gpu_kernels.cu, train_kaggle_lse.cu, train_kaggle_qkv.cu and
generate_routed.c into <out dir>)
"""
import os
import sys

GUARD_FIRST, GUARD_LAST = 253, 489        # gpu_kernels.cu: the attention section

SHRINK_EDITS = [
    ('#include "gpu_kernels.h"\n',
     '#include "gpu_kernels.h"\n#define ATTN_OMIT_MACRO_DROPINS\n#include "attn_b200.h"\n'),
    ("static void alloc_acts(void) {\n",
     "static void alloc_acts(void) {\n    if (attn_set_probs_mode(ATTN_PROBS_LSE) != ATTN_OK) exit(1);\n"),
    ("long PB = (long)B_SIZE * N_HEADS * T_SIZE * T_SIZE;",
     "long PB = (long)B_SIZE * N_HEADS * T_SIZE;"),
    ("s_Dbuf = dmalloc((long)B_SIZE * N_HEADS * T_SIZE * T_SIZE);",
     "s_Dbuf = dmalloc(2L * B_SIZE * N_HEADS * T_SIZE);"),
]

# train_kaggle.cu:152-154
QKV_OLD = (
    "        gemm_nn(a_ln1[l], W(o_Wq[l]), W(o_bq[l]), a_q[l], M, DIM, DIM);\n"
    "        gemm_nn(a_ln1[l], W(o_Wk[l]), W(o_bk[l]), a_k[l], M, DIM, DIM);\n"
    "        gemm_nn(a_ln1[l], W(o_Wv[l]), W(o_bv[l]), a_v[l], M, DIM, DIM);\n")
QKV_NEW = ("        attn_qkv_proj(a_ln1[l], W(o_Wq[l]), W(o_Wk[l]), W(o_Wv[l]), W(o_bq[l]), W(o_bk[l]), W(o_bv[l]),\n"
           "                      a_q[l], a_k[l], a_v[l], M, DIM, DIM);\n")

# generate.c:129 (the scale) .. 152 (the end of the per-head loop)
GEN_LOOP_FIRST = "    const float scale = 1.0f / sqrtf((float)DH);\n"
GEN_LOOP_END = "\n    matvec(s_proj, s_att, w->Wo, w->bo, D, D);\n"
GEN_CALL = "    attn_cached_attention_host_ex(s_q, g_kc[l], g_vc[l], s_att, pos, H, DH, D, BLK);\n"


def guard_gpu_kernels(text):
    lines = text.split("\n")
    if not lines[GUARD_FIRST - 1].startswith("/* ========================== attention"):
        raise ValueError("gpu_kernels.cu: the attention section does not start at line %d" % GUARD_FIRST)
    if not (lines[GUARD_LAST - 1] == "}" and "embeddings" in lines[GUARD_LAST + 1]):
        raise ValueError("gpu_kernels.cu: the attention section does not end at line %d" % GUARD_LAST)
    lines.insert(GUARD_LAST, "#endif /* ATTN_EXTERNAL */")
    lines.insert(GUARD_FIRST - 1, "#ifndef ATTN_EXTERNAL")
    return "\n".join(lines)


def shrink_trainer(text):
    for old, new in SHRINK_EDITS:
        if text.count(old) != 1:
            raise ValueError("train_kaggle.cu: expected one %r" % old)
        text = text.replace(old, new)
    return text


def fuse_qkv(text):
    """Applied to the output of shrink_trainer (which includes attn_b200.h)."""
    if text.count(QKV_OLD) != 1:
        raise ValueError("train_kaggle.cu: the three Q, K, V gemm_nn calls were not found together")
    return text.replace(QKV_OLD, QKV_NEW)


def route_generate(text):
    if text.count(GEN_LOOP_FIRST) != 1 or text.count(GEN_LOOP_END) != 1:
        raise ValueError("generate.c: the attention loop of block() was not found")
    a = text.index(GEN_LOOP_FIRST)
    b = text.index(GEN_LOOP_END)
    loop = text[a:b]
    if "for (int h = 0; h < H; h++)" not in loop or "s_att + off" not in loop:
        raise ValueError("generate.c: unexpected text between the scale and the Wo product")
    text = text[:a] + GEN_CALL + text[b:]
    inc = '#include "tokenizer.h"\n'
    if text.count(inc) != 1:
        raise ValueError("generate.c: expected one tokenizer include")
    return text.replace(inc, inc + '#include "attn_b200.h"\n')


def main(argv):
    ref, out = argv[1], argv[2]
    os.makedirs(out, exist_ok=True)

    def rd(name):
        with open(os.path.join(ref, name)) as f:
            return f.read()

    def wr(name, text):
        with open(os.path.join(out, name), "w") as f:
            f.write(text)

    wr("gpu_kernels.cu", guard_gpu_kernels(rd("gpu_kernels.cu")))
    wr("train_kaggle_lse.cu", shrink_trainer(rd("train_kaggle.cu")))
    wr("train_kaggle_qkv.cu", fuse_qkv(shrink_trainer(rd("train_kaggle.cu"))))
    wr("generate_routed.c", route_generate(rd("generate.c")))


if __name__ == "__main__":
    main(sys.argv)
