// The block executor's small ops on device memory: the ops the reference's
// gate claims next to its matmuls (src/xdna-exec.cpp:97-131) and runs on
// host threads, row by row (run_rows, :253-346; the rope table, :194-239).
// Each is HBM-bound elementwise or row-reduction work: grid-stride loops,
// float4 accesses where rows allow, one block per row for RMS_NORM.
// Arithmetic follows the reference's float expressions; transcendental
// functions are CUDA's accurate ones (no fast-math intrinsics).
#include "zest_b200.h"
#include "zest_device.cuh"
#include "zest_internal.h"

#include <algorithm>
#include <cmath>

namespace zest {

namespace {

int blocks_for(int64_t n, int threads) {
    const int64_t b = (n + threads - 1) / threads;
    return (int) (b < 148 * 32 ? (b > 0 ? b : 1) : 148 * 32);
}

// y = x * (1 / sqrt(mean(x^2) + eps)) per row of d (ggml RMS_NORM)
__global__ void rms_norm_kernel(const float *__restrict__ x, int64_t rows, int64_t d, float eps, float *__restrict__ y) {
    __shared__ float part[32];
    for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
        const float *xr = x + r * d;
        const float sc = 1.0f / sqrtf(block_sumsq(xr, d, part) / (float) d + eps);
        for (int64_t j = threadIdx.x; j < d; j += blockDim.x) y[r * d + j] = __fmul_rn(xr[j], sc);
    }
}

// y = x * w (a row broadcast over every row), x + b (same shape or a bias row)
template <int OP>  // 0 mul row, 1 add same shape, 2 add bias row
__global__ void binary_kernel(const float *__restrict__ x, const float *__restrict__ b, int64_t n, int64_t d,
                              float *__restrict__ y) {
    for (int64_t i = blockIdx.x * (int64_t) blockDim.x + threadIdx.x; i < n; i += (int64_t) gridDim.x * blockDim.x) {
        if (OP == 0) y[i] = __fmul_rn(x[i], b[i % d]);
        else if (OP == 1) y[i] = __fadd_rn(x[i], b[i]);
        else y[i] = __fadd_rn(x[i], b[i % d]);
    }
}

__global__ void scale_kernel(const float *__restrict__ x, int64_t n, float s, float bias, float *__restrict__ y) {
    for (int64_t i = blockIdx.x * (int64_t) blockDim.x + threadIdx.x; i < n; i += (int64_t) gridDim.x * blockDim.x)
        y[i] = __fadd_rn(__fmul_rn(x[i], s), bias);
}

__device__ __forceinline__ float act(int kind, float g) {
    switch (kind) {
        case 2: return g / (1.0f + expf(-g));                                                    // SiLU
        case 1: return 0.5f * g * (1.0f + tanhf(0.7978845608f * g * (1.0f + 0.044715f * g * g)));  // GELU (tanh)
        case 4: return 0.5f * g * (1.0f + erff(g * 0.7071067812f));                              // GELU (erf)
        case 5: return g / (1.0f + expf(-1.702f * g));                                           // GELU (quick)
        default: return g > 0.0f ? g : 0.0f;                                                     // ReLU
    }
}

__global__ void glu_kernel(int kind, const float *__restrict__ g, int64_t gs, const float *__restrict__ u, int64_t us,
                           int64_t rows, int64_t f, float *__restrict__ y) {
    const int64_t n = rows * f;
    for (int64_t i = blockIdx.x * (int64_t) blockDim.x + threadIdx.x; i < n; i += (int64_t) gridDim.x * blockDim.x) {
        const int64_t r = i / f, j = i % f;
        const float gv = g[r * gs + j], uv = u[r * us + j];
        y[i] = kind == 0 ? (gv > 0.0f ? gv * uv : 0.0f) : act(kind, gv) * uv;
    }
}

struct rope_consts {
    float corr0, corr1, theta_scale, freq_scale, ext_factor, attn_factor, log_scale;
    int n_dims;
};

// One token's cos/sin row: theta multiplied by theta_scale pair after pair,
// as the reference builds its table (and ggml-cpu its cache).
__global__ void rope_table_kernel(const int32_t *__restrict__ pos, int64_t T, const float *__restrict__ ff,
                                  rope_consts k, float *__restrict__ table) {
    for (int64_t t = blockIdx.x * (int64_t) blockDim.x + threadIdx.x; t < T; t += (int64_t) gridDim.x * blockDim.x) {
        float theta = (float) pos[t];
        float *cs = table + t * k.n_dims;
        for (int p = 0; p < k.n_dims / 2; p++) {
            const float extrap = ff ? theta / ff[p] : theta;
            float th = k.freq_scale * extrap, mscale = k.attn_factor;
            if (k.ext_factor != 0.0f) {
                const float y = ((float) p - k.corr0) / fmaxf(0.001f, k.corr1 - k.corr0);
                const float ramp_mix = (1.0f - fminf(1.0f, fmaxf(0.0f, y))) * k.ext_factor;
                th = th * (1.0f - ramp_mix) + extrap * ramp_mix;
                mscale *= 1.0f + 0.1f * k.log_scale;
            }
            cs[2 * p] = cosf(th) * mscale;
            cs[2 * p + 1] = sinf(th) * mscale;
            theta *= k.theta_scale;
        }
    }
}

// x [T][heads][d]: each (token, head, pair) rotated; dims past n_dims copied.
__global__ void rope_kernel(const float *__restrict__ x, int64_t T, int64_t heads, int64_t d, int n_dims, int neox,
                            const float *__restrict__ table, float *__restrict__ y) {
    const int64_t half = d / 2 + (d & 1), n = T * heads * half;
    const int64_t off_n = neox ? n_dims / 2 : 1;
    for (int64_t i = blockIdx.x * (int64_t) blockDim.x + threadIdx.x; i < n; i += (int64_t) gridDim.x * blockDim.x) {
        const int64_t row = i / half, q = i % half, t = row / heads;
        const float *src = x + row * d;
        float *dst = y + row * d;
        if (2 * q < n_dims) {
            const int64_t ic = neox ? q : 2 * q;
            const float c = table[t * n_dims + 2 * q], s = table[t * n_dims + 2 * q + 1];
            const float x0 = src[ic], x1 = src[ic + off_n];
            dst[ic] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
            dst[ic + off_n] = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
        } else {
            const int64_t j = n_dims + (2 * q - n_dims);
            if (j < d) dst[j] = src[j];
            if (j + 1 < d) dst[j + 1] = src[j + 1];
        }
    }
}

}  // namespace

}  // namespace zest

using namespace zest;

// bf16 -> f32, exact: 8 values a thread (one 16-byte load, two 16-byte
// stores), grid-stride; the ragged tail one value a thread.
__global__ void widen_bf16_kernel(const uint16_t *__restrict__ src, int64_t n, float *__restrict__ dst) {
    const int64_t n8 = n / 8;
    for (int64_t i = blockIdx.x * (int64_t) blockDim.x + threadIdx.x; i < n8; i += (int64_t) gridDim.x * blockDim.x) {
        const uint4 h = reinterpret_cast<const uint4 *>(src)[i];
        float4 *d = reinterpret_cast<float4 *>(dst) + 2 * i;
        d[0] = make_float4(__uint_as_float(h.x << 16), __uint_as_float(h.x & 0xffff0000u), __uint_as_float(h.y << 16),
                           __uint_as_float(h.y & 0xffff0000u));
        d[1] = make_float4(__uint_as_float(h.z << 16), __uint_as_float(h.z & 0xffff0000u), __uint_as_float(h.w << 16),
                           __uint_as_float(h.w & 0xffff0000u));
    }
    const int64_t t = 8 * n8 + blockIdx.x * (int64_t) blockDim.x + threadIdx.x;
    if (t < n) dst[t] = __uint_as_float((uint32_t) src[t] << 16);
}

extern "C" {

int zest_rms_norm(const float *x, int64_t rows, int64_t d, float eps, float *y, void *stream) {
    if (rows <= 0) return 0;
    if (d <= 0) return set_error("zest_rms_norm: empty rows");
    rms_norm_kernel<<<(int) (rows < 148 * 16 ? rows : 148 * 16), 256, 0, (cudaStream_t) stream>>>(x, rows, d, eps, y);
    return check_launch("zest_rms_norm");
}

int zest_mul_row(const float *x, const float *w, int64_t rows, int64_t d, float *y, void *stream) {
    const int64_t n = rows * d;
    if (n <= 0) return 0;
    binary_kernel<0><<<blocks_for(n, 256), 256, 0, (cudaStream_t) stream>>>(x, w, n, d, y);
    return check_launch("zest_mul_row");
}

int zest_add(const float *x, const float *b, int bias_row, int64_t rows, int64_t d, float *y, void *stream) {
    const int64_t n = rows * d;
    if (n <= 0) return 0;
    if (bias_row) binary_kernel<2><<<blocks_for(n, 256), 256, 0, (cudaStream_t) stream>>>(x, b, n, d, y);
    else binary_kernel<1><<<blocks_for(n, 256), 256, 0, (cudaStream_t) stream>>>(x, b, n, d, y);
    return check_launch("zest_add");
}

int zest_widen_bf16(const uint16_t *src, int64_t n, float *dst, void *stream) {
    if (n <= 0) return 0;
    if (!src || !dst || ((uintptr_t) src & 15) || ((uintptr_t) dst & 15))
        return set_error("zest_widen_bf16: src and dst must be 16-byte aligned");
    widen_bf16_kernel<<<blocks_for(std::max<int64_t>(1, n / 8), 256), 256, 0, (cudaStream_t) stream>>>(src, n, dst);
    return check_launch("zest_widen_bf16");
}

int zest_scale(const float *x, int64_t n, float s, float bias, float *y, void *stream) {
    if (n <= 0) return 0;
    scale_kernel<<<blocks_for(n, 256), 256, 0, (cudaStream_t) stream>>>(x, n, s, bias, y);
    return check_launch("zest_scale");
}

int zest_glu(int kind, const float *g, int64_t g_stride, const float *u, int64_t u_stride, int64_t rows, int64_t f,
             float *y, void *stream) {
    if (kind != ZEST_GLU_REGLU && kind != ZEST_GLU_GEGLU && kind != ZEST_GLU_SWIGLU && kind != ZEST_GLU_GEGLU_ERF &&
        kind != ZEST_GLU_GEGLU_QUICK)
        return set_error("zest_glu: unsupported GLU kind");
    if (rows * f <= 0) return 0;
    glu_kernel<<<blocks_for(rows * f, 256), 256, 0, (cudaStream_t) stream>>>(kind, g, g_stride, u, u_stride, rows, f,
                                                                            y);
    return check_launch("zest_glu");
}

// ggml_rope_yarn_corr_dims: the published YaRN correction range, in the
// same float operations.
static float corr_dim(int n_dims, int n_ctx_orig, float n_rot, float base) {
    return (float) n_dims * logf((float) n_ctx_orig / (n_rot * 2.0f * (float) 3.14159265358979323846)) / (2.0f * logf(base));
}

int zest_rope_table(const int32_t *pos, int64_t T, int n_dims, int n_ctx_orig, const float *par, const float *ff,
                    float *table, void *stream) {
    if (T <= 0) return 0;
    if (n_dims <= 0 || n_dims % 2 || !par) return set_error("zest_rope_table: n_dims must be even and positive");
    rope_consts k;
    const float start = floorf(corr_dim(n_dims, n_ctx_orig, par[4], par[0]));
    const float end = ceilf(corr_dim(n_dims, n_ctx_orig, par[5], par[0]));
    k.corr0 = start > 0.0f ? start : 0.0f;
    k.corr1 = end < (float) (n_dims - 1) ? end : (float) (n_dims - 1);
    k.theta_scale = powf(par[0], -2.0f / (float) n_dims);
    k.freq_scale = par[1];
    k.ext_factor = par[2];
    k.attn_factor = par[3];
    k.log_scale = logf(1.0f / par[1]);
    k.n_dims = n_dims;
    rope_table_kernel<<<blocks_for(T, 128), 128, 0, (cudaStream_t) stream>>>(pos, T, ff, k, table);
    return check_launch("zest_rope_table");
}

int zest_rope(const float *x, int64_t T, int64_t heads, int64_t d, int n_dims, int mode, const float *table, float *y,
              void *stream) {
    if (mode != ZEST_ROPE_NORMAL && mode != ZEST_ROPE_NEOX) return set_error("zest_rope: unsupported mode");
    if (n_dims <= 0 || n_dims % 2 || n_dims > d) return set_error("zest_rope: bad n_dims");
    const int64_t n = T * heads * (d / 2 + (d & 1));
    if (n <= 0) return 0;
    rope_kernel<<<blocks_for(n, 256), 256, 0, (cudaStream_t) stream>>>(x, T, heads, d, n_dims,
                                                                      mode == ZEST_ROPE_NEOX, table, y);
    return check_launch("zest_rope");
}

}  // extern "C"
