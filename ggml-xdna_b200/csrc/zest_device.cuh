// Device-side building blocks shared by the three kernels: the bfp16 block
// codec (bit-exact with the reference's AVX2 packer), the bfp16 tile
// addressing, and thin PTX wrappers for mbarriers, TMA and tcgen05.
//
// Reference: src/npu/bfp16_pack.cpp:85-144 (codec), :172-186 (offsets).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace zest {

constexpr int BLOCK_BYTES = 9;  // one exponent byte + eight int8 mantissas
constexpr int TILE_M = 128;     // A: rows per tile (bfp16_tiling::m)
constexpr int TILE_K = 64;      // values along K per tile (bfp16_tiling::k)
constexpr int TILE_N = 64;      // B: rows per tile (bfp16_tiling::n)
constexpr int TILE_COLS = 8;    // B: array columns (bfp16_tiling::cols)
constexpr int SUB_BYTES = 16 * (TILE_K / 8) * BLOCK_BYTES;  // 16 rows x one k tile = 1152 B, contiguous

// Error bits a kernel can raise in the caller's device flag word.
enum : unsigned {
    ERR_NOT_FINITE = 1u,  // an output was NaN or infinite (xdna-npu.cpp:59-67)
    ERR_TIMEOUT = 2u,     // a bounded wait ran out
};

__device__ __forceinline__ uint32_t f2u(float f) { return __float_as_uint(f); }
__device__ __forceinline__ float u2f(uint32_t u) { return __uint_as_float(u); }

// A row's sum of squares over a block of threads, in a fixed order: each
// thread a strided partial of fused multiply-adds, then an xor tree within
// each warp and another over the warps' partials (part: 32 floats of shared
// memory). RMS_NORM and the kernels that fuse it share this, so they agree
// bit for bit. Every thread of the block must call it.
__device__ __forceinline__ float block_sumsq(const float *__restrict__ xr, int64_t d, float *part) {
    float ss = 0.0f;
    for (int64_t j = threadIdx.x; j < d; j += blockDim.x) ss = __fmaf_rn(xr[j], xr[j], ss);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
    __syncthreads();
    float v = 0.0f;
    if (threadIdx.x < 32) {
        v = threadIdx.x < (blockDim.x >> 5) ? part[threadIdx.x] : 0.0f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    }
    __syncthreads();
    if (threadIdx.x == 0) part[0] = v;
    __syncthreads();
    v = part[0];
    __syncthreads();  // part[] is free for the next row
    return v;
}

// bf16 bits of x, rounded to nearest even (NaN stays NaN).
__device__ __forceinline__ uint16_t bf16_bits_rne(float x) {
    uint32_t u = __float_as_uint(x);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t) ((u | 0x00400000u) >> 16);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t) (u >> 16);
}

// One block of eight floats -> nine bytes, as bfp16_encode_block's AVX2 path
// (bfp16_pack.cpp:85-114, compiled with -mavx2 in the reference's builds):
//  * exponent byte = the largest biased float exponent of the eight;
//  * when 2^(133 - e) is a normal float (e >= 6), q = rne(x * 2^(133 - e)),
//    with x86 cvtps2dq's answer for NaN/Inf (0x80000000, clamping to -128);
//  * all (signed) zeros -> nine zero bytes;
//  * e <= 5: the scalar path, rne(ldexp(x, 133 - e)), same clamp.
// Also returns the decoded values as bf16 bits (exactly representable).
__device__ __forceinline__ void encode_block(const float (&x)[8], uint8_t (&out)[9], uint32_t (&bf)[4]) {
    uint32_t mx = 0, any = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const uint32_t u = f2u(x[i]);
        mx = max(mx, (u >> 23) & 0xffu);
        any |= u & 0x7fffffffu;
    }
    int q[8];
    if (mx >= 6 && mx <= 200) {
        // every value finite and the block's quantum Q = 2^(e - 133) in the
        // normal or subnormal range: rounding x * 2^(133 - e) to an integer,
        // nearest even, is rounding x to a multiple of Q, which one add and
        // one subtract of C = 1.5 * 2^23 * Q do exactly (|x| < 2^7 Q, far
        // inside the 2^22 Q the method needs); then q <= 127 is d <= 127 Q
        // (x / Q > -128 always, so -128 never clamps). d is q * Q exactly,
        // the decoded value, and has at most 8 significant bits.
        const float C = u2f(((mx + 17u) << 23) | 0x400000u);  // 1.5 * 2^(mx - 110)
        const float top = u2f((mx << 23) | 0x7E0000u);        // 127 * 2^(mx - 133)
        const float scale = u2f((260u - mx) << 23);           // 2^(133 - mx)
        uint32_t h[8];
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const float d = fminf(__fsub_rn(__fadd_rn(x[i], C), C), top);
            h[i] = f2u(d) >> 16;
            q[i] = __float2int_rz(__fmul_rn(d, scale));
        }
        out[0] = (uint8_t) mx;
#pragma unroll
        for (int i = 0; i < 8; i++) out[1 + i] = (uint8_t) (int8_t) q[i];
#pragma unroll
        for (int i = 0; i < 4; i++) bf[i] = h[2 * i] | (h[2 * i + 1] << 16);
        return;
    }
    if (mx >= 6) {
        const float scale = u2f((260u - mx) << 23);
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const float p = __fmul_rn(x[i], scale);
            int v = ((f2u(x[i]) >> 23) & 0xffu) == 0xffu ? -128 : __float2int_rn(p);
            q[i] = min(127, max(-128, v));
        }
    } else if (any == 0) {
        mx = 0;
#pragma unroll
        for (int i = 0; i < 8; i++) q[i] = 0;
    } else {
        // x * 2^(133 - e), e <= 5: two exact power-of-two steps
        const float s1 = u2f((127u + 64u) << 23);                 // 2^64
        const float s2 = u2f((127u + (133u - mx) - 64u) << 23);   // 2^(69 - e)
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const float p = __fmul_rn(__fmul_rn(x[i], s1), s2);
            q[i] = min(127, max(-128, __float2int_rn(p)));
        }
    }
    out[0] = (uint8_t) mx;
#pragma unroll
    for (int i = 0; i < 8; i++) out[1 + i] = (uint8_t) (int8_t) q[i];
    // decoded value q * 2^(e - 133), as bf16 bits
    uint32_t h[8];
    if (mx >= 7) {
        const float scale = u2f((mx - 6u) << 23);  // 2^(e - 133)
#pragma unroll
        for (int i = 0; i < 8; i++) h[i] = f2u(__fmul_rn((float) q[i], scale)) >> 16;
    } else {
        const float s1 = u2f((mx + 58u) << 23);   // 2^(e - 69)
        const float s2 = u2f((127u - 64u) << 23); // 2^-64
#pragma unroll
        for (int i = 0; i < 8; i++) h[i] = f2u(__fmul_rn(__fmul_rn((float) q[i], s1), s2)) >> 16;
    }
#pragma unroll
    for (int i = 0; i < 4; i++) bf[i] = h[2 * i] | (h[2 * i + 1] << 16);
}

// The same encoding with a block split over two lanes (lane ^ 1 holds the
// other four values): the block's max exponent and its all-zero test are
// combined with one warp shuffle each. Returns this lane's four int8
// mantissas packed in a word, the block's exponent byte, and the four
// decoded values as bf16 bits. Every lane of the warp must call it.
__device__ __forceinline__ void encode_half_block(const float4 x4, uint32_t &q_packed, uint32_t &exp_byte,
                                                  uint2 &bf) {
    const float x[4] = { x4.x, x4.y, x4.z, x4.w };
    uint32_t mx = 0, any = 0;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const uint32_t u = f2u(x[i]);
        mx = max(mx, (u >> 23) & 0xffu);
        any |= u & 0x7fffffffu;
    }
    mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    any |= __shfl_xor_sync(0xffffffffu, any, 1);
    int q[4];
    if (mx >= 6) {
        const float scale = u2f((260u - mx) << 23);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int v = ((f2u(x[i]) >> 23) & 0xffu) == 0xffu ? -128 : __float2int_rn(__fmul_rn(x[i], scale));
            q[i] = min(127, max(-128, v));
        }
    } else if (any == 0) {
        mx = 0;
#pragma unroll
        for (int i = 0; i < 4; i++) q[i] = 0;
    } else {
        const float s1 = u2f((127u + 64u) << 23), s2 = u2f((127u + (133u - mx) - 64u) << 23);
#pragma unroll
        for (int i = 0; i < 4; i++) q[i] = min(127, max(-128, __float2int_rn(__fmul_rn(__fmul_rn(x[i], s1), s2))));
    }
    exp_byte = mx;
    q_packed = (uint32_t) (q[0] & 0xff) | ((uint32_t) (q[1] & 0xff) << 8) | ((uint32_t) (q[2] & 0xff) << 16) |
               ((uint32_t) (q[3] & 0xff) << 24);
    uint32_t h[4];
    if (mx >= 7) {
        const float scale = u2f((mx - 6u) << 23);
#pragma unroll
        for (int i = 0; i < 4; i++) h[i] = f2u(__fmul_rn((float) q[i], scale)) >> 16;
    } else {
        const float s1 = u2f((mx + 58u) << 23), s2 = u2f((127u - 64u) << 23);
#pragma unroll
        for (int i = 0; i < 4; i++) h[i] = f2u(__fmul_rn(__fmul_rn((float) q[i], s1), s2)) >> 16;
    }
    bf = make_uint2(h[0] | (h[1] << 16), h[2] | (h[3] << 16));
}

// Where block column cb of row rr sits inside one tile, in blocks:
// 16-row pairs, then block columns, then the 16 rows (bfp16_pack.cpp:172-175).
__host__ __device__ __forceinline__ int64_t in_tile(int64_t rr, int64_t cb) {
    return ((rr / 16) * (TILE_K / 8) + cb % (TILE_K / 8)) * 16 + rr % 16;
}

// Byte offset of the 1152-byte run holding rows [r0, r0+16) (r0 % 16 == 0)
// of k tile kt, in an A operand of K columns (bfp16_a_offset, :177-180).
__host__ __device__ __forceinline__ int64_t a_run_offset(int64_t r0, int64_t kt, int64_t K) {
    const int64_t nk = K / TILE_K;
    const int64_t tile = (r0 / TILE_M) * nk + kt;
    return (tile * TILE_M * (TILE_K / 8) + in_tile(r0 % TILE_M, 0)) * BLOCK_BYTES;
}

// The same in a B operand of N rows (N % 512 == 0) (bfp16_b_offset, :182-186).
__host__ __device__ __forceinline__ int64_t b_run_offset(int64_t r0, int64_t kt, int64_t N, int64_t K) {
    const int64_t per_col = N / TILE_N / TILE_COLS, nk = K / TILE_K, g = r0 / TILE_N;
    const int64_t tile = ((g % TILE_COLS) * per_col + g / TILE_COLS) * nk + kt;
    return (tile * TILE_N * (TILE_K / 8) + in_tile(r0 % TILE_N, 0)) * BLOCK_BYTES;
}

// ---------------------------------------------------------------------------
// PTX wrappers (sm_100a)
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t) __cvta_generic_to_shared(p);
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Waits for the phase of `parity` to complete, for at most `limit_ns`, or
// until *abort (when given) is set by another thread of the block. False if
// it gave up.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity, volatile int *abort,
                                                  uint64_t limit_ns) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (uint32_t it = 0;; it++) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 63u) == 63u) {
            if (abort && *abort) return false;
            if (global_ns() - t0 > limit_ns) return false;
        }
    }
}

// Spins until *flag == want (acquire, GPU scope) or limit_ns passes (false).
__device__ __forceinline__ bool flag_wait_bounded(const int *flag, int want, volatile int *abort, uint64_t limit_ns) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
    if (v == want) return true;
    const uint64_t t0 = global_ns();
    for (uint32_t it = 0;; it++) {
        asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
        if (v == want) return true;
        if ((it & 15u) == 15u) {
            if (abort && *abort) return false;
            if (global_ns() - t0 > limit_ns) return false;
        }
        __nanosleep(64);
    }
}

__device__ __forceinline__ void flag_release(int *flag, int v) {
    asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(flag), "r"(v) : "memory");
}

// Adds to the value at a multicast address in every GPU bound to it: the
// NVSwitch performs the reduction (NVLink SHARP). Relaxed, system scope.
__device__ __forceinline__ void multimem_red_add_v4(float *mc, float a, float b, float c, float d) {
    asm volatile("multimem.red.relaxed.sys.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc), "f"(a), "f"(b),
                 "f"(c), "f"(d)
                 : "memory");
}

// Stores to the address in every GPU bound to the multicast object (the
// NVSwitch replicates the write). Relaxed, system scope.
__device__ __forceinline__ void multimem_st_v4(float *mc, float a, float b, float c, float d) {
    asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc), "f"(a), "f"(b), "f"(c),
                 "f"(d)
                 : "memory");
}

__device__ __forceinline__ void multimem_st(float *mc, float a) {
    asm volatile("multimem.st.relaxed.sys.global.f32 [%0], %1;" ::"l"(mc), "f"(a) : "memory");
}

__device__ __forceinline__ void multimem_red_add(float *mc, float a) {
    asm volatile("multimem.red.relaxed.sys.global.add.f32 [%0], %1;" ::"l"(mc), "f"(a) : "memory");
}

// A barrier among the `n` threads (a multiple of 32) that name barrier `id`.
__device__ __forceinline__ void named_barrier(int id, int n) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

// 2D TMA tile load into shared memory, completing on `bar` (no multicast).
__device__ __forceinline__ void tma_load_2d(void *dst, const void *tmap, uint64_t *bar, int32_t c0, int32_t c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
        ::"r"(smem_u32(dst)), "l"(tmap), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
        : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const void *tmap) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

// --- tcgen05 ---------------------------------------------------------------

__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (bf16 in, fp32 accumulate)
__device__ __forceinline__ void tc_mma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrives on `bar` once every tcgen05 op this thread issued so far is done.
__device__ __forceinline__ void tc_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i gets lane (base + i).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// The wait for a load into r issued earlier and left in flight: r is tied
// to the wait, so no use of it moves above the wait.
__device__ __forceinline__ void tmem_ld_wait(uint32_t (&r)[32]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                   "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                   "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
                 :
                 : "memory");
}

// --- CTA pairs (a cluster of 2 sharing one tcgen05 MMA) -----------------------

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// Every thread of both CTAs; a hardware barrier, not a spin.
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// The address of the same shared-memory offset in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_to_rank(const void *p, uint32_t rank) {
    uint32_t out;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(smem_u32(p)), "r"(rank));
    return out;
}

// Arrive on a barrier given by its shared::cluster address (possibly the peer's).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

// 2D TMA tile load by one CTA of a pair into its own shared memory, whose
// completion counts on the barrier at `bar_cluster_addr` (the pair leader's).
// No multicast.
__device__ __forceinline__ void tma_load_2d_pair(void *dst, const void *tmap, uint32_t bar_cluster_addr, int32_t c0,
                                                 int32_t c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%3, %4}], [%2];"
        ::"r"(smem_u32(dst)), "l"(tmap), "r"(bar_cluster_addr), "r"(c0), "r"(c1)
        : "memory");
}

// An L2 policy that marks every line a copy touches evict-first: for data
// read or written once (the streamed operand, the outputs), so it does not
// push the operand that every wave re-reads out of L2.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// tma_load_2d_pair with an L2 cache policy.
__device__ __forceinline__ void tma_load_2d_pair_hint(void *dst, const void *tmap, uint32_t bar_cluster_addr,
                                                      int32_t c0, int32_t c1, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint "
        "[%0], [%1, {%3, %4}], [%2], %5;"
        ::"r"(smem_u32(dst)), "l"(tmap), "r"(bar_cluster_addr), "r"(c0), "r"(c1), "l"(policy)
        : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t *dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// D[tmem of both CTAs] (+)= A[both CTAs' smem] * B[both CTAs' smem]^T, M=256
// across the pair; issued by the pair leader.
__device__ __forceinline__ void tc_mma_bf16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                                 uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrives on the barrier at the same offset in every CTA of `cta_mask` once
// the leader's tcgen05 ops so far are done.
__device__ __forceinline__ void tc_commit_pair_mc(uint64_t *bar, uint16_t cta_mask) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;"
        ::"r"(smem_u32(bar)), "h"(cta_mask)
        : "memory");
}

// Arrives on the barrier at `bar_cluster_addr` once the pair's tcgen05 ops
// this thread issued so far are done.
__device__ __forceinline__ void tc_commit_pair(uint32_t bar_cluster_addr) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar_cluster_addr)
                 : "memory");
}

// --- bulk tensor stores (shared -> global), for the GEMM epilogue -------------

// Makes this thread's shared-memory writes visible to the TMA engine.
__device__ __forceinline__ void fence_proxy_async_shared() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// 2D TMA tile store from shared memory; the engine clips rows and columns
// outside the tensor. No reduction, no multicast.
__device__ __forceinline__ void tma_store_2d(const void *tmap, const void *src, int32_t c0, int32_t c1) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(tmap),
                 "r"(smem_u32(src)), "r"(c0), "r"(c1)
                 : "memory");
}

// tma_store_2d with an L2 cache policy.
__device__ __forceinline__ void tma_store_2d_hint(const void *tmap, const void *src, int32_t c0, int32_t c1,
                                                  uint64_t policy) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group.L2::cache_hint [%0, {%2, %3}], [%1], %4;"
                 ::"l"(tmap), "r"(smem_u32(src)), "r"(c0), "r"(c1), "l"(policy)
                 : "memory");
}

__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

// Until at most N committed store groups still read shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

// Until every committed store group has completed.
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Orders this thread's async-proxy (TMA) and generic-proxy accesses to
// global memory, e.g. completed TMA stores before a system-scope fence.
__device__ __forceinline__ void fence_proxy_async_global() {
    asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Shared-memory matrix descriptor for a K-major bf16 tile written by TMA
// with 128-byte swizzle: rows of 128 B (64 values), 8-row atoms of 1 KB.
__device__ __forceinline__ uint64_t sw128_desc(const void *tile) {
    const uint64_t addr = smem_u32(tile);
    return ((addr & 0x3ffffu) >> 4)      // start address
           | (1ull << 16)                // leading byte offset (unused with swizzle)
           | ((1024ull >> 4) << 32)      // stride byte offset: next 8-row atom
           | (1ull << 46)                // descriptor version (sm_100)
           | (2ull << 61);               // SWIZZLE_128B
}

}  // namespace zest
