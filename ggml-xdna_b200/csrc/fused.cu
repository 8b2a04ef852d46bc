// The block executor's ops folded into the kernels beside them. The
// reference runs each claimed small op as its own host pass over the rows
// (run_rows, src/xdna-exec.cpp:253-346) and encodes the next matmul's input
// in yet another (encode_row, src/xdna-npu.cpp:511-515); here one pass reads
// the row once and writes what the next step consumes.
//
//   zest_pack_rms_norm  RMS_NORM, the MUL by its weight row, and K2's pack:
//                       f32 rows in, the GEMM's bf16 A operand out (and the
//                       f32 result only when something else reads it)
//   zest_norm_rope      per-head RMS_NORM, MUL and ROPE (Qwen3's q/k path):
//                       f32 in, f32 and/or bf16 out
//
// Both give the bits of the separate kernels: the row sums share
// block_sumsq's order (or, per head, an order the tests pin against the
// oracle), and every multiply and add is an explicitly rounded one.
#include "zest_b200.h"
#include "zest_device.cuh"
#include "zest_internal.h"

namespace zest {

namespace {

constexpr int NP_THREADS = 256;

// One block per row (grid-stride): the row's sum of squares as
// rms_norm_kernel forms it, then 8-value blocks scaled, multiplied by the
// weight row, written as f32 (optional) and as the bf16 copy of their bfp16
// encoding. Rows in [T, m_pad) of the operand are zero, as the pack's.
__global__ void __launch_bounds__(NP_THREADS) norm_pack_kernel(const float *__restrict__ x, int64_t T, int64_t K,
                                                               int64_t ldx, float eps, const float *__restrict__ w,
                                                               float *__restrict__ y, int64_t ldy, int64_t m_pad,
                                                               uint16_t *__restrict__ a, int64_t lda) {
    __shared__ float part[32];
    for (int64_t r = blockIdx.x; r < m_pad; r += gridDim.x) {
        uint16_t *ar = a + r * lda;
        if (r >= T) {
            for (int64_t j = threadIdx.x * 8; j < K; j += NP_THREADS * 8)
                *reinterpret_cast<uint4 *>(ar + j) = make_uint4(0, 0, 0, 0);
            continue;
        }
        const float *xr = x + r * ldx;
        const float sc = 1.0f / sqrtf(block_sumsq(xr, K, part) / (float) K + eps);
        for (int64_t j = threadIdx.x * 8; j < K; j += NP_THREADS * 8) {
            const float4 p0 = *reinterpret_cast<const float4 *>(xr + j);
            const float4 p1 = *reinterpret_cast<const float4 *>(xr + j + 4);
            float v[8] = { p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w };
#pragma unroll
            for (int i = 0; i < 8; i++) v[i] = __fmul_rn(v[i], sc);
            if (w) {
                const float4 w0 = *reinterpret_cast<const float4 *>(w + j);
                const float4 w1 = *reinterpret_cast<const float4 *>(w + j + 4);
                const float wv[8] = { w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w };
#pragma unroll
                for (int i = 0; i < 8; i++) v[i] = __fmul_rn(v[i], wv[i]);
            }
            if (y) {
                float *yr = y + r * ldy + j;
                *reinterpret_cast<float4 *>(yr) = make_float4(v[0], v[1], v[2], v[3]);
                *reinterpret_cast<float4 *>(yr + 4) = make_float4(v[4], v[5], v[6], v[7]);
            }
            uint8_t enc[9];
            uint32_t bf[4];
            encode_block(v, enc, bf);
            *reinterpret_cast<uint4 *>(ar + j) = make_uint4(bf[0], bf[1], bf[2], bf[3]);
        }
    }
}

constexpr int NR_WARPS = 8, NR_MAX_D = 256;

// One warp per (token, head) row of d: the row's RMS norm and weight, staged
// in shared memory, then each value rotated with its partner (NeoX: the two
// halves of the first n_dims; normal: adjacent pairs), as rope_kernel does.
__global__ void __launch_bounds__(NR_WARPS * 32) norm_rope_kernel(const float *__restrict__ x, int64_t T, int64_t H,
                                                                  int64_t d, float eps, const float *__restrict__ w,
                                                                  int n_dims, int neox, const float *__restrict__ table,
                                                                  float *__restrict__ y, uint16_t *__restrict__ y16) {
    __shared__ float buf[NR_WARPS][NR_MAX_D];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float *row = buf[warp];
    const int64_t rows = T * H;
    for (int64_t r = (int64_t) blockIdx.x * NR_WARPS + warp; r < rows; r += (int64_t) gridDim.x * NR_WARPS) {
        const float *xr = x + r * d;
        float ss = 0.0f;
        for (int64_t j = lane; j < d; j += 32) ss = __fmaf_rn(xr[j], xr[j], ss);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float sc = 1.0f / sqrtf(ss / (float) d + eps);
        for (int64_t j = lane; j < d; j += 32) {
            float v = __fmul_rn(xr[j], sc);
            if (w) v = __fmul_rn(v, w[j]);
            row[j] = v;
        }
        __syncwarp();
        const float *cs = table + (r / H) * n_dims;
        const int half = n_dims / 2;
        for (int64_t j = lane; j < d; j += 32) {
            float out = row[j];
            if (j < n_dims) {
                const bool first = neox ? j < half : (j & 1) == 0;
                const int p = neox ? (first ? (int) j : (int) j - half) : (int) (j >> 1);
                const int64_t partner = neox ? (first ? j + half : j - half) : (j ^ 1);
                const float c = cs[2 * p], s = cs[2 * p + 1];
                const float x0 = first ? row[j] : row[partner], x1 = first ? row[partner] : row[j];
                out = first ? __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s))
                            : __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
            }
            if (y) y[r * d + j] = out;
            if (y16) y16[r * d + j] = bf16_bits_rne(out);
        }
        __syncwarp();
    }
}

int grid_of(int64_t units, int per_sm) {
    const int64_t cap = 148ll * per_sm;
    return (int) (units < 1 ? 1 : (units < cap ? units : cap));
}

}  // namespace

}  // namespace zest

using namespace zest;

extern "C" {

int zest_pack_rms_norm(const float *x, int64_t T, int64_t K, int64_t ldx, float eps, const float *w, float *y,
                       int64_t ldy, int64_t m_pad, uint16_t *a_bf16, int64_t lda, void *stream) {
    if (T < 0 || K <= 0 || K % 8 || m_pad < T || m_pad % 128 || ldx < K || ldx % 4 || ((uintptr_t) x & 15) ||
        ((uintptr_t) w & 15) || !a_bf16 || lda < K || lda % 8 || ((uintptr_t) a_bf16 & 15) ||
        (y && (ldy < K || ldy % 4 || ((uintptr_t) y & 15))))
        return set_error("zest_pack_rms_norm: K a multiple of 8, m_pad of 128 covering T, rows 16-byte aligned");
    if (m_pad == 0) return 0;
    norm_pack_kernel<<<grid_of(m_pad, 16), NP_THREADS, 0, (cudaStream_t) stream>>>(x, T, K, ldx, eps, w, y, ldy,
                                                                                    m_pad, a_bf16, lda);
    return check_launch("zest_pack_rms_norm");
}

int zest_norm_rope(const float *x, int64_t T, int64_t heads, int64_t d, float eps, const float *w, int n_dims,
                   int mode, const float *table, float *y, uint16_t *y_bf16, void *stream) {
    if (mode != ZEST_ROPE_NORMAL && mode != ZEST_ROPE_NEOX) return set_error("zest_norm_rope: unsupported mode");
    if (d <= 0 || d > NR_MAX_D || n_dims <= 0 || n_dims % 2 || n_dims > d || !table)
        return set_error("zest_norm_rope: head size at most 256, n_dims even and within it");
    const int64_t rows = T * heads;
    if (rows <= 0) return 0;
    norm_rope_kernel<<<grid_of((rows + NR_WARPS - 1) / NR_WARPS, 8), NR_WARPS * 32, 0, (cudaStream_t) stream>>>(
        x, T, heads, d, eps, w, n_dims, mode == ZEST_ROPE_NEOX, table, y, y_bf16);
    return check_launch("zest_norm_rope");
}

}  // extern "C"
