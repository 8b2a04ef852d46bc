// K2 (activation pack) and K1 (weight conversion): memory-bound kernels that
// write the reference's bfp16 operand layout byte for byte, plus the exact
// bf16 expansion of the same values that the tensor-core GEMM reads.
//
// Reference: activation encode src/xdna-npu.cpp:406-420,476-515 with
// bfp16_a_row (src/npu/bfp16_pack.h:82-84); weight conversion
// src/xdna-npu.cpp:339-390 (ggml to_float, then bfp16_pack_b,
// bfp16_interleave_gate_up).
//
// In the reference layout the 128 blocks of 16 rows x one 64-wide k tile are
// one contiguous 1152-byte run (a 16-row pair, all 8 block columns), so both
// kernels encode their bytes into shared memory and store whole runs as
// aligned 16-byte vectors.
#include "zest_device.cuh"
#include "zest_internal.h"

#include <cuda_fp16.h>

namespace zest {

__device__ __forceinline__ void store_run(uint8_t *dst, const uint8_t *stage, int tid, int nthreads) {
    const uint4 *s = reinterpret_cast<const uint4 *>(stage);
    uint4 *d = reinterpret_cast<uint4 *>(dst);
    for (int i = tid; i < SUB_BYTES / 16; i += nthreads) d[i] = s[i];
}

// ---------------------------------------------------------------------------
// K2: f32 activations [T][K] (row stride ldx) -> A operand
// ---------------------------------------------------------------------------

// A work unit is 16 rows x 256 columns (4 k tiles). Warp w streams rows w
// and w + 8, each as two 512-byte segments of 128 floats: every load
// instruction is one fully coalesced 512-byte run. Lane l holds values
// [4l, 4l + 4) of a segment, so lanes 2j and 2j+1 share block j and combine
// its max exponent with one shuffle. All four loads are issued before any
// encoding. The bfp16 bytes go through shared memory to leave as the four
// tiles' 1152-byte runs.
constexpr int PACK_THREADS = 256;

template <bool BYTES, bool BF16>
__global__ void __launch_bounds__(PACK_THREADS) pack_activations_kernel(const float *__restrict__ x, int64_t T,
                                                                        int64_t K, int64_t ldx, int64_t m_pad,
                                                                        uint8_t *__restrict__ a_bytes,
                                                                        uint16_t *__restrict__ a_bf16, int64_t ldb) {
    constexpr int W = 256;  // columns per unit
    __shared__ __align__(16) uint8_t stage[BYTES ? (W / TILE_K) * SUB_BYTES : 16];
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int nkt = (int) (K / TILE_K), ngroups = (nkt + 3) / 4;
    const int64_t units = (m_pad / 16) * ngroups;
    for (int64_t u = blockIdx.x; u < units; u += gridDim.x) {
        const int64_t r0 = (u / ngroups) * 16;
        const int c0 = (int) (u % ngroups) * W, width = min(W, (int) K - c0);  // a multiple of 64
        float4 ld[2][2];
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const int64_t r = r0 + warp + 8 * h;
#pragma unroll
            for (int s = 0; s < 2; s++) {
                const int col = c0 + s * 128 + 4 * lane;
                // rows past the prompt are zeros (xdna-npu.cpp:416-418)
                ld[h][s] = (r < T && s * 128 + 4 * lane < width)
                               ? __ldg(reinterpret_cast<const float4 *>(x + r * ldx + col))
                               : make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const int rr = warp + 8 * h;
#pragma unroll
            for (int s = 0; s < 2; s++) {
                const int cu = s * 128 + 4 * lane;  // column within the unit
                uint32_t q, e;
                uint2 bf;
                encode_half_block(ld[h][s], q, e, bf);
                if (cu >= width) continue;
                if (BF16) *reinterpret_cast<uint2 *>(a_bf16 + (r0 + rr) * ldb + c0 + cu) = bf;
                if (BYTES) {
                    const int kt = cu / TILE_K, cb = (cu % TILE_K) / 8;
                    uint8_t *blk = stage + kt * SUB_BYTES + (cb * 16 + rr) * BLOCK_BYTES;
                    const int off = (lane & 1) ? 5 : 1;
                    if (!(lane & 1)) blk[0] = (uint8_t) e;
#pragma unroll
                    for (int j = 0; j < 4; j++) blk[off + j] = (uint8_t) (q >> (8 * j));
                }
            }
        }
        if (BYTES) {
            __syncthreads();
            for (int i = 0; i < width / TILE_K; i++)
                store_run(a_bytes + a_run_offset(r0, c0 / TILE_K + i, K), stage + i * SUB_BYTES, threadIdx.x,
                          PACK_THREADS);
            __syncthreads();
        }
    }
}

// ---------------------------------------------------------------------------
// K1: GGUF weight rows -> B operand
// ---------------------------------------------------------------------------

__device__ uint32_t g_iq3s_grid[512];

struct quant_info {
    int qk;          // values per quant block
    int block_bytes; // bytes per quant block
};

__host__ __device__ constexpr quant_info quant_of(int type) {
    switch (type) {
        case TYPE_F32: return { 1, 4 };
        case TYPE_F16: return { 1, 2 };
        case TYPE_Q8_0: return { 32, 34 };
        case TYPE_Q4_K: return { 256, 144 };
        case TYPE_Q6_K: return { 256, 210 };
        case TYPE_IQ3_S: return { 256, 110 };
    }
    return { 0, 0 };
}

__device__ __forceinline__ float ld_half(const uint8_t *p) {
    return __half2float(__ushort_as_half((unsigned short) (p[0] | (p[1] << 8))));
}

// Dequantises the 8 values at column `col` (col % 8 == 0) of one row, whose
// raw bytes from the start of the unit's first quant block sit at `seg`;
// `col` counts from that same block. Float operations are written with
// explicit roundings in ggml's order, so no multiply-add is contracted.
template <int TYPE>
__device__ __forceinline__ void dequant8(const uint8_t *seg, int col, float (&y)[8]) {
    if constexpr (TYPE == TYPE_F32) {
#pragma unroll
        for (int i = 0; i < 8; i++) {
            uint32_t u;
            memcpy(&u, seg + (col + i) * 4, 4);
            y[i] = __uint_as_float(u);
        }
    } else if constexpr (TYPE == TYPE_F16) {
#pragma unroll
        for (int i = 0; i < 8; i++) y[i] = ld_half(seg + (col + i) * 2);
    } else if constexpr (TYPE == TYPE_Q8_0) {
        // y = qs * d (ggml dequantize_row_q8_0)
        const uint8_t *b = seg + (col / 32) * 34;
        const float d = ld_half(b);
        const int8_t *qs = reinterpret_cast<const int8_t *>(b + 2 + col % 32);
#pragma unroll
        for (int i = 0; i < 8; i++) y[i] = __fmul_rn((float) qs[i], d);
    } else if constexpr (TYPE == TYPE_Q4_K) {
        // sub-block j of 32: y = (d*sc_j) * q - (dmin*m_j) (ggml dequantize_row_q4_K)
        const uint8_t *b = seg + (col / 256) * 144;
        const int idx = col % 256, j = idx / 32, l0 = idx % 32;
        const float d = ld_half(b), dmin = ld_half(b + 2);
        const uint8_t *sc = b + 4, *q = b + 16 + (j / 2) * 32;
        int s, m;
        if (j < 4) {
            s = sc[j] & 63;
            m = sc[j + 4] & 63;
        } else {
            s = (sc[j + 4] & 0xF) | ((sc[j - 4] >> 6) << 4);
            m = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
        }
        const float d1 = __fmul_rn(d, (float) s), m1 = __fmul_rn(dmin, (float) m);
        const int sh = (j & 1) * 4;
#pragma unroll
        for (int i = 0; i < 8; i++) y[i] = __fsub_rn(__fmul_rn(d1, (float) ((q[l0 + i] >> sh) & 0xF)), m1);
    } else if constexpr (TYPE == TYPE_Q6_K) {
        // y = (d*sc) * (q6 - 32) (ggml dequantize_row_q6_K)
        const uint8_t *b = seg + (col / 256) * 210;
        const int idx = col % 256, n = idx / 128, r = idx % 128, quarter = r / 32, l0 = r % 32;
        const float d = ld_half(b + 208);
        const int8_t *sc = reinterpret_cast<const int8_t *>(b + 192) + n * 8;
        const uint8_t *ql = b + n * 64 + (quarter & 1) * 32, *qh = b + 128 + n * 32;
        const float ds = __fmul_rn(d, (float) sc[l0 / 16 + 2 * quarter]);
        const int lsh = quarter >= 2 ? 4 : 0, hsh = 2 * quarter;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const int q = (((ql[l0 + i] >> lsh) & 0xF) | (((qh[l0 + i] >> hsh) & 3) << 4)) - 32;
            y[i] = __fmul_rn(ds, (float) q);
        }
    } else if constexpr (TYPE == TYPE_IQ3_S) {
        // y = (d*(1+2s)) * grid * sign (ggml dequantize_row_iq3_s)
        const uint8_t *b = seg + (col / 256) * 110;
        const int idx = col % 256, ib32 = idx / 32, l = (idx % 32) / 8;
        const float d = ld_half(b);
        const uint8_t *qs = b + 2 + ib32 * 8, qh = b[66 + ib32], sg = b[74 + ib32 * 4 + l];
        const int sc = (ib32 & 1) ? (b[106 + ib32 / 2] >> 4) : (b[106 + ib32 / 2] & 0xF);
        const float db = __fmul_rn(d, (float) (1 + 2 * sc));
        const uint32_t g1 = g_iq3s_grid[qs[2 * l] | (((qh >> (2 * l)) & 1) << 8)];
        const uint32_t g2 = g_iq3s_grid[qs[2 * l + 1] | (((qh >> (2 * l + 1)) & 1) << 8)];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            y[i] = __fmul_rn(__fmul_rn(db, (float) ((g1 >> (8 * i)) & 0xFF)), (sg >> i) & 1 ? -1.0f : 1.0f);
            y[i + 4] = __fmul_rn(__fmul_rn(db, (float) ((g2 >> (8 * i)) & 0xFF)), (sg >> (i + 4)) & 1 ? -1.0f : 1.0f);
        }
    }
}

// Source of output row r of the B operand: plain (row src_row0 + r of src0,
// zeros past n_rows) or a fused gate/up pair (bfp16_interleave_gate_up: 8
// gate rows, then the 8 up rows that pair with them; zeros past F).
struct row_source {
    const uint8_t *src0, *src1;
    int64_t n_rows;   // real rows (N, or F when fused)
    int64_t src_row0; // first source row (N-sharding)
    int64_t row_bytes;
    int64_t total_bytes0, total_bytes1;  // bytes readable at src0 / src1
    int fused;
};

__device__ __forceinline__ const uint8_t *source_row(const row_source &s, int64_t r, int64_t &limit,
                                                     const uint8_t *&base) {
    int64_t i = r;
    base = s.src0;
    limit = s.total_bytes0;
    if (s.fused) {
        i = (r / 16) * 8 + r % 8;
        if (r % 16 >= 8) {
            base = s.src1;
            limit = s.total_bytes1;
        }
    }
    if (i >= s.n_rows) return nullptr;
    return base + (s.src_row0 + i) * s.row_bytes;
}

// Copies the 16-byte aligned span around bytes [p, p + n) to the aligned
// slot `dst` in 128-bit loads (the tensor base is 16-byte aligned; rows need
// not be), never reading at or past base + limit. Returns where p landed:
// dst + (p mod 16).
__device__ __forceinline__ int stage_bytes(uint8_t *dst, const uint8_t *base, const uint8_t *p, int n, int64_t limit,
                                           int lane, int nlanes) {
    const uintptr_t a0 = (uintptr_t) p & ~(uintptr_t) 15, a1 = ((uintptr_t) p + n + 15) & ~(uintptr_t) 15;
    const uintptr_t end = (uintptr_t) base + (uintptr_t) limit;
    const int chunks = (int) ((a1 - a0) / 16);
    for (int i = lane; i < chunks; i += nlanes) {
        const uintptr_t at = a0 + (uintptr_t) i * 16;
        if (at + 16 <= end) {
            *reinterpret_cast<uint4 *>(dst + i * 16) = __ldg(reinterpret_cast<const uint4 *>(at));
        } else {
            for (int j = 0; j < 16; j++)
                if (at + j < end) dst[i * 16 + j] = *reinterpret_cast<const uint8_t *>(at + j);
        }
    }
    return (int) ((uintptr_t) p - a0);
}

template <int TYPE, int W>
__global__ void __launch_bounds__(128) convert_weight_kernel(row_source src, int64_t n_pad, int64_t K,
                                                             uint8_t *__restrict__ b_bytes,
                                                             uint16_t *__restrict__ b_bf16) {
    constexpr quant_info qi = quant_of(TYPE);
    constexpr int SEG = W / qi.qk * qi.block_bytes;   // raw bytes of one row's unit
    constexpr int SLOT = (SEG + 30 + 15) / 16 * 16;    // aligned staging slot per row (SEG + misalignment)
    constexpr int KT = W / TILE_K;                       // k tiles per unit
    __shared__ __align__(16) uint8_t raw[16 * SLOT];
    __shared__ __align__(16) uint8_t stage[KT * SUB_BYTES];
    __shared__ int head[16];
    const int tid = threadIdx.x;
    const int64_t nw = K / W, units = (n_pad / 16) * nw;
    for (int64_t u = blockIdx.x; u < units; u += gridDim.x) {
        const int64_t r0 = (u / nw) * 16, w0 = (u % nw) * W;
        // stage the unit's raw bytes: 8 threads per row
        {
            const int row = tid / 8, lane = tid % 8;  // 16 rows x 8 threads = the whole block
            int64_t limit;
            const uint8_t *base;
            const uint8_t *rp = source_row(src, r0 + row, limit, base);
            if (rp) {
                const int h = stage_bytes(raw + row * SLOT, base, rp + (w0 / qi.qk) * qi.block_bytes, SEG, limit, lane, 8);
                if (lane == 0) head[row] = h;
            }
        }
        __syncthreads();
        // a warp per row, a lane per 8-value block: each warp's bf16 store is
        // one contiguous run of the row (512 bytes when W = 256)
        const int warp = tid / 32, lane = tid % 32;
        for (int row = warp; row < 16; row += 4) {
            int64_t limit;
            const uint8_t *base;
            const bool real = source_row(src, r0 + row, limit, base) != nullptr;
            for (int cb = lane; cb < W / 8; cb += 32) {
                const int col = cb * 8, kt = col / TILE_K, c = (col % TILE_K) / 8;
                float v[8];
                if (real) {
                    dequant8<TYPE>(raw + row * SLOT + head[row], col, v);
                } else {
#pragma unroll
                    for (int i = 0; i < 8; i++) v[i] = 0.0f;  // padding rows (xdna-npu.cpp:372, pad_n)
                }
                uint8_t enc[9];
                uint32_t bf[4];
                encode_block(v, enc, bf);
                if (b_bf16)
                    *reinterpret_cast<uint4 *>(b_bf16 + (r0 + row) * K + w0 + col) =
                        make_uint4(bf[0], bf[1], bf[2], bf[3]);
                if (b_bytes) {
                    // the tile's order: 16-row pair, then block column, then row
                    uint8_t *s = stage + kt * SUB_BYTES + (c * 16 + row) * BLOCK_BYTES;
#pragma unroll
                    for (int i = 0; i < 9; i++) s[i] = enc[i];
                }
            }
        }
        __syncthreads();
        if (b_bytes)
            for (int kt = 0; kt < KT; kt++)
                store_run(b_bytes + b_run_offset(r0, w0 / TILE_K + kt, n_pad, K), stage + kt * SUB_BYTES, tid, 128);
        __syncthreads();
    }
}

// ---------------------------------------------------------------------------
// launchers
// ---------------------------------------------------------------------------

static int grid_for(int64_t units, int per_sm) {
    static int sms = 0;
    if (!sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (sms <= 0) sms = 148;
    }
    const int64_t cap = (int64_t) sms * per_sm;
    return (int) (units < cap ? units : cap);
}

int launch_pack_activations(const float *x, int64_t T, int64_t K, int64_t ldx, int64_t m_pad, uint8_t *a_bytes,
                            uint16_t *a_bf16, int64_t ldb, cudaStream_t st) {
    if (K % TILE_K || m_pad % TILE_M || m_pad < T || T < 0 || ldx < K || ldx % 4 || ((uintptr_t) x & 15))
        return set_error("pack_activations: K must be a multiple of 64, m_pad a multiple of 128 covering T, "
                         "and rows 16-byte aligned");
    if (a_bf16 && (ldb < K || ldb % 8 || ((uintptr_t) a_bf16 & 15)))
        return set_error("pack_activations: bf16 rows must be 16-byte aligned");
    const int64_t units = (m_pad / 16) * ((K / TILE_K + 3) / 4);
    if (units == 0) return 0;
    const int grid = grid_for(units, 8);
    if (a_bytes && a_bf16)
        pack_activations_kernel<true, true><<<grid, PACK_THREADS, 0, st>>>(x, T, K, ldx, m_pad, a_bytes, a_bf16, ldb);
    else if (a_bytes)
        pack_activations_kernel<true, false><<<grid, PACK_THREADS, 0, st>>>(x, T, K, ldx, m_pad, a_bytes, a_bf16, ldb);
    else if (a_bf16)
        pack_activations_kernel<false, true><<<grid, PACK_THREADS, 0, st>>>(x, T, K, ldx, m_pad, a_bytes, a_bf16, ldb);
    else
        return 0;
    return check_launch("pack_activations");
}

int set_iq3s_grid(const uint32_t *grid512) {
    if (cudaMemcpyToSymbol(g_iq3s_grid, grid512, 512 * sizeof(uint32_t)) != cudaSuccess)
        return set_error("cannot load the IQ3_S codebook");
    return 0;
}

template <int TYPE, int W>
static void launch_convert_t(const row_source &s, int64_t n_pad, int64_t K, uint8_t *b, uint16_t *h, cudaStream_t st) {
    const int64_t units = (n_pad / 16) * (K / W);
    convert_weight_kernel<TYPE, W><<<grid_for(units, 16), 128, 0, st>>>(s, n_pad, K, b, h);
}

int launch_convert_weight(int type, const void *src0, const void *src1, int fused, int64_t n_rows, int64_t src_row0,
                          int64_t src_rows_total, int64_t K, int64_t n_pad, uint8_t *b_bytes, uint16_t *b_bf16,
                          cudaStream_t st) {
    const quant_info qi = quant_of(type);
    if (!qi.qk) return set_error("convert_weight: unsupported weight type");
    if (K % TILE_K || K % qi.qk || n_pad % (TILE_N * TILE_COLS) || ((uintptr_t) src0 & 15) ||
        (fused && ((uintptr_t) src1 & 15)))
        return set_error("convert_weight: K must be a multiple of 64 and of the quant block, n_pad of 512, "
                         "sources 16-byte aligned");
    if ((fused ? 2 * n_rows : n_rows) > n_pad) return set_error("convert_weight: n_pad too small");
    if (type == TYPE_IQ3_S && !iq3s_grid_loaded()) return set_error("convert_weight: no IQ3_S codebook loaded");
    row_source s;
    s.src0 = (const uint8_t *) src0;
    s.src1 = (const uint8_t *) (fused ? src1 : src0);
    s.n_rows = n_rows;
    s.src_row0 = src_row0;
    s.row_bytes = K / qi.qk * qi.block_bytes;
    s.total_bytes0 = src_rows_total * s.row_bytes;
    s.total_bytes1 = src_rows_total * s.row_bytes;
    s.fused = fused;
    const bool wide = K % 256 == 0;
    switch (type) {
        case TYPE_F32:
            if (wide) launch_convert_t<TYPE_F32, 256>(s, n_pad, K, b_bytes, b_bf16, st);
            else launch_convert_t<TYPE_F32, 64>(s, n_pad, K, b_bytes, b_bf16, st);
            break;
        case TYPE_F16:
            if (wide) launch_convert_t<TYPE_F16, 256>(s, n_pad, K, b_bytes, b_bf16, st);
            else launch_convert_t<TYPE_F16, 64>(s, n_pad, K, b_bytes, b_bf16, st);
            break;
        case TYPE_Q8_0:
            if (wide) launch_convert_t<TYPE_Q8_0, 256>(s, n_pad, K, b_bytes, b_bf16, st);
            else launch_convert_t<TYPE_Q8_0, 64>(s, n_pad, K, b_bytes, b_bf16, st);
            break;
        case TYPE_Q4_K: launch_convert_t<TYPE_Q4_K, 256>(s, n_pad, K, b_bytes, b_bf16, st); break;
        case TYPE_Q6_K: launch_convert_t<TYPE_Q6_K, 256>(s, n_pad, K, b_bytes, b_bf16, st); break;
        case TYPE_IQ3_S: launch_convert_t<TYPE_IQ3_S, 256>(s, n_pad, K, b_bytes, b_bf16, st); break;
    }
    return check_launch("convert_weight");
}

}  // namespace zest
