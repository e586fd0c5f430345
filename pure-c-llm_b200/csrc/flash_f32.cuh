// flash_f32.cuh -- tile machinery shared by the fp32-arithmetic flash kernels
// (forward and backward).  These are the precision path: every product and
// sum is an fp32 FFMA on the CUDA cores, so results track the reference's
// fp32 loops (train.c:339-407) to ~1e-6 relative.
//
// Tile geometry: 64 x 64 score tiles, 128 threads as a 16 x 8 grid (ty, tx).
// Thread (ty, tx) owns score rows {ty + 16 i | i < 4} and columns
// {tx + 8 j | j < 8}; output rows are the same four, output columns the
// float4 groups {4 tx + 32 c}.  Shared tiles are row-major with a 4-float pad
// so that the eight tx lanes reading rows tx, tx+8, ... land in distinct bank
// groups.
#pragma once
#include "common.cuh"
#include "sm100.cuh"

namespace attn {

constexpr int kFBM = 64;          // query rows per tile
constexpr int kFBN = 64;          // key rows per tile
constexpr int kFThreads = 128;

template <int D> struct FTile {
    static constexpr int LD = D + 4;             // padded row length (floats)
    static constexpr int FLOATS = kFBM * LD;     // one 64-row tile
};

__device__ __forceinline__ void cp_async16(float *smem_dst, const float *gsrc) {
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem_dst);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gsrc));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N> __device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

// Stages rows [row0, row0+64) of a (rows x stride) activation slice into a
// padded fp32 tile; rows at or beyond `nrows` are zero-filled.  fp32 sources
// go through cp.async (caller commits/waits); bf16 sources are widened in
// registers.
template <typename T, int D>
__device__ __forceinline__ void load_tile(float *dst, const T *src, long long stride, int row0,
                                          int nrows, int tid)
{
    constexpr int CPR = D / 4;                   // 16-byte (4-element) chunks per row
    constexpr int LD = FTile<D>::LD;
#pragma unroll 4
    for (int idx = tid; idx < kFBM * CPR; idx += kFThreads) {
        const int r = idx / CPR, c = idx % CPR;
        float *d = dst + r * LD + c * 4;
        const int gr = row0 + r;
        if (gr < nrows) {
            if constexpr (sizeof(T) == 4) {
                cp_async16(d, reinterpret_cast<const float *>(src) + (long long)gr * stride + c * 4);
            } else {
                *reinterpret_cast<float4 *>(d) = load4(src + (long long)gr * stride + c * 4);
            }
        } else {
            *reinterpret_cast<float4 *>(d) = make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
}

// acc[i][j] += A[ty+16i][:] . B[tx+8j][:] over D, A and B padded row-major tiles.
template <int D>
__device__ __forceinline__ void tile_qkT(float (&acc)[4][8], const float *A, const float *B,
                                         int ty, int tx)
{
    constexpr int LD = FTile<D>::LD;
#pragma unroll 2
    for (int k = 0; k < D; k += 4) {
        float4 a[4], b[8];
#pragma unroll
        for (int i = 0; i < 4; i++) a[i] = *reinterpret_cast<const float4 *>(A + (ty + 16 * i) * LD + k);
#pragma unroll
        for (int j = 0; j < 8; j++) b[j] = *reinterpret_cast<const float4 *>(B + (tx + 8 * j) * LD + k);
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 8; j++) {
                acc[i][j] = fmaf(a[i].x, b[j].x, acc[i][j]);
                acc[i][j] = fmaf(a[i].y, b[j].y, acc[i][j]);
                acc[i][j] = fmaf(a[i].z, b[j].z, acc[i][j]);
                acc[i][j] = fmaf(a[i].w, b[j].w, acc[i][j]);
            }
    }
}

// Writes a 64x64 weight tile W[row][col] (owned as acc[i][j] at row ty+16i,
// col tx+8j) into Wt[col][4 ty + i] -- column-major with the four rows of a
// thread adjacent, so the product pass reads them with one 16-byte load.
__device__ __forceinline__ void store_weights_T(float *Wt, const float (&w)[4][8], int ty, int tx)
{
#pragma unroll
    for (int j = 0; j < 8; j++)
        *reinterpret_cast<float4 *>(Wt + (tx + 8 * j) * (kFBM + 4) + 4 * ty) =
            make_float4(w[0][j], w[1][j], w[2][j], w[3][j]);
}

// out[i][c] += sum_n W[ty+16i][n] * M[n][4tx + 32(c/4) + c%4]; W given as Wt
// from store_weights_T, M a padded row-major 64 x D tile.  The products run on
// f32x2 pairs (two adjacent output columns per fma.rn.f32x2, each lane rounded
// as fmaf would), so a warp issues half the FMA instructions.
template <int D>
__device__ __forceinline__ void tile_wM(float (&out)[4][D / 8], const float *Wt, const float *M,
                                        int ty, int tx)
{
    constexpr int LD = FTile<D>::LD;
#pragma unroll 4
    for (int n = 0; n < kFBN; n++) {
        const float4 w = *reinterpret_cast<const float4 *>(Wt + n * (kFBM + 4) + 4 * ty);
        const uint64_t wb[4] = {sm100::f2(w.x, w.x), sm100::f2(w.y, w.y), sm100::f2(w.z, w.z), sm100::f2(w.w, w.w)};
#pragma unroll
        for (int c = 0; c < D / 32; c++) {
            const float4 m = *reinterpret_cast<const float4 *>(M + n * LD + 4 * tx + 32 * c);
            const uint64_t mlo = sm100::f2(m.x, m.y), mhi = sm100::f2(m.z, m.w);
#pragma unroll
            for (int i = 0; i < 4; i++) {
                uint64_t lo = sm100::f2(out[i][4 * c + 0], out[i][4 * c + 1]);
                uint64_t hi = sm100::f2(out[i][4 * c + 2], out[i][4 * c + 3]);
                lo = sm100::fma2(wb[i], mlo, lo);
                hi = sm100::fma2(wb[i], mhi, hi);
                sm100::f2_split(lo, out[i][4 * c + 0], out[i][4 * c + 1]);
                sm100::f2_split(hi, out[i][4 * c + 2], out[i][4 * c + 3]);
            }
        }
    }
}

// Reductions over the 8 tx lanes that share a row (lanes differ in bits 0-2).
__device__ __forceinline__ float row_max8(float v) {
    v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 1));
    v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 2));
    v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 4));
    return v;
}
__device__ __forceinline__ float row_sum8(float v) {
    v += __shfl_xor_sync(0xffffffffu, v, 1);
    v += __shfl_xor_sync(0xffffffffu, v, 2);
    v += __shfl_xor_sync(0xffffffffu, v, 4);
    return v;
}

}  // namespace attn
