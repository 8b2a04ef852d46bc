// K3: the bfp16 GEMM on the 5th-generation tensor cores.
//
// C[M x N] = A[M x K] * B[N x K]^T, where A and B hold bfp16-decoded values
// (every bfp16 value is exact in bf16), so a bf16 x bf16 -> fp32 tcgen05 MMA
// computes the reference's products exactly and only the fp32 summation
// order differs (mm_paired, kernels/bfp16_gemm/aie_kernels/aie2p/
// mm_bfp_acc.cc:44-100). The epilogue applies the reference's output modes
// (out_epilogue, :258-278), un-tiles to ggml's row-major [M][N] as
// bfp16_c_row / bfp16_c16_row do (src/npu/bfp16_pack.cpp:188-229), and
// raises a device flag on any NaN/Inf result (all_finite,
// src/xdna-npu.cpp:59-67).
//
// Two kernels, both persistent (one CTA, or one CTA pair, per SM) and warp-
// specialised:
//
// gemm_bf16_tc_pair_kernel<BN_T> (the default; M > 128): a cluster of two
// CTAs on one 256 x BN_T output tile with cta_group::2 MMAs (M=256 split
// 128 + 128 across the pair, N=BN_T, K=16 per instruction). 192 threads:
//   warp 0      TMA producer: this CTA's 128x64 A half and BN_T/2 x 64 B half,
//               128-byte swizzle, into a shared-memory ring (stages sized to
//               fill ~192 KB), completing on the leader CTA's barrier
//   warp 1      TMEM allocator (cta_group::2) and, in the leader, the single-
//               thread MMA issuer; its commits multicast to both CTAs
//   warps 2-5   epilogue: tcgen05.ld 32 lanes x 32 columns, the output mode,
//               then a double-buffered, swizzled 32x32 staging tile per warp
//               stored by TMA (direct stores where TMA cannot: misaligned
//               output rows)
// The tile loop walks up to 4 weights sharing A (q, k, v; gate, up) as one
// space of N tiles: a grouped launch is one kernel, no tails between them.
// The walk's order (rows, columns or groups of 8 M blocks) is chosen per
// launch to keep the re-read operand in L2. A second instance,
// <BN_T, true>, adds stream-K: the last wave's tiles cut into runs of
// k-blocks across all pairs, partial sums through a per-CTA workspace
// (used by default for K >= 8192). The epilogue also fuses the residual ADD,
// SwiGLU's packed output for the next GEMM, and, for tensor-parallel
// partials, multimem.red into an NVLink multicast buffer.
//
// gemm_bf16_tc_kernel (M <= 128, and ZEST_GEMM_PAIR=0): one CTA on a 128x256
// tile, 192 threads: warp 0 TMA, warp 1 TMEM + MMA (M=128, N=256), warps 2-5
// epilogue with direct stores.
//
// Two 256-column accumulators (all 512 TMEM columns) let the epilogue of one
// tile overlap the MMAs of the next. Every wait is bounded; on timeout the
// kernel raises ERR_TIMEOUT, drains its own copies and MMAs, frees TMEM and
// returns. No TMA load uses cluster multicast: each CTA loads its own halves.
#include "zest_device.cuh"
#include "zest_internal.h"

#include <cuda.h>
#include <mutex>
#include <cudaTypedefs.h>

namespace zest {

namespace {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;
constexpr int B_BYTES = BN * BK * 2;
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int ACC_COLS = BN;
constexpr int TMEM_COLS = 2 * ACC_COLS;
constexpr int NUM_THREADS = 192;
constexpr int NUM_BARRIERS = 2 * STAGES + 5;
constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + NUM_BARRIERS * 8 + 16;
constexpr uint64_t WAIT_LIMIT_NS = 1000000000ull;  // 1 s
constexpr int GROUP_M = 8;

// kind::f16 instruction descriptor: fp32 accumulate, bf16 A and B, both
// K-major, N=256, M=128.
constexpr uint32_t IDESC = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t) (BN >> 3) << 17) |
                           ((uint32_t) (BM >> 4) << 24);

struct gemm_params {
    int64_t M, N, K, ldc;
    int64_t n_out;  // output columns (N, or the real F for SwiGLU)
    float *c;
    unsigned *err;
    int mode, num_m, num_n, num_k;
    int tma_store;  // pair kernel: the epilogue stores through shared memory with TMA
    const float *resid;  // c = resid + result (fp32 and bf16 modes), or null
    int64_t ldr;
    uint16_t *a_next;    // SwiGLU: the result's bfp16-rounded bf16 copy, the next GEMM's A, or null
    int64_t lda_next;
    float *c_mc;         // or null: the results added (multimem.red) into a multicast buffer [M][ldc]
    int mc_store;        // with c_mc: the results stored (multimem.st) into every copy instead
    int n_peers;         // pair kernel with TMA stores: each tile also stored into this many peers' copies
    int n_c16;           // pair kernel: each tile stored in bf16 into this many copies (bf16 mode)
};

__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int &mb, int &nb) {
    const int per_group = GROUP_M * num_n;
    const int g = t / per_group, first_m = g * GROUP_M;
    const int gsz = min(num_m - first_m, GROUP_M);
    const int r = t % per_group;
    mb = first_m + r % gsz;
    nb = r / gsz;
}

__device__ __forceinline__ uint32_t not_finite(float v) {
    return (__float_as_uint(v) & 0x7f800000u) == 0x7f800000u;
}

// Two floats rounded to bf16, nearest even, by the hardware's paired
// conversion (a NaN comes back as a NaN), and widened back to floats.
__device__ __forceinline__ void bf16_round2(float &x, float &y) {
    uint32_t p;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(p) : "f"(y), "f"(x));
    x = __uint_as_float(p << 16);
    y = __uint_as_float(p & 0xffff0000u);
}

// Whether any of 32 values is NaN or infinite, without a branch: x * 0 is 0
// for every finite x and NaN otherwise.
__device__ __forceinline__ uint32_t any_not_finite(const float (&o)[32]) {
    float c0 = 0.0f, c1 = 0.0f;
#pragma unroll
    for (int i = 0; i < 32; i += 2) {
        c0 = __fmaf_rn(o[i], 0.0f, c0);
        c1 = __fmaf_rn(o[i + 1], 0.0f, c1);
    }
    const float c = c0 + c1;
    return c != c;
}

// o[i] = resid[row][col0 + i] + o[i] for the columns the output holds (the
// ADD that follows o and down in a layer, fused: an f32 add of the same
// operands as the separate op).
__device__ __forceinline__ void add_residual(const gemm_params &p, float (&o)[32], int64_t row, int64_t col0) {
    const float *src = p.resid + row * p.ldr + col0;
    if (col0 + 32 <= p.n_out && (p.ldr % 4) == 0 && ((uintptr_t) p.resid & 15) == 0) {
#pragma unroll
        for (int i = 0; i < 32; i += 4) {
            const float4 q = *reinterpret_cast<const float4 *>(src + i);
            o[i] = __fadd_rn(q.x, o[i]);
            o[i + 1] = __fadd_rn(q.y, o[i + 1]);
            o[i + 2] = __fadd_rn(q.z, o[i + 2]);
            o[i + 3] = __fadd_rn(q.w, o[i + 3]);
        }
    } else {
#pragma unroll
        for (int i = 0; i < 32; i++)
            if (col0 + i < p.n_out) o[i] = __fadd_rn(src[i], o[i]);
    }
}

// Writes one thread's 32 accumulator columns [col0, col0+32) of row `row`.
__device__ __forceinline__ uint32_t store_chunk(const gemm_params &p, const uint32_t (&r)[32], int64_t row,
                                                int64_t col0) {
    uint32_t bad = 0;
    if (row >= p.M) return 0;
    if (p.mode == MODE_SWIGLU) {
        // columns: 8 gate, 8 up, 8 gate, 8 up -> 16 outputs
        float o[16];
#pragma unroll
        for (int h = 0; h < 2; h++)
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const float g = __uint_as_float(r[h * 16 + i]), u = __uint_as_float(r[h * 16 + 8 + i]);
                const float s = 1.0f / (1.0f + expf(-g));
                o[h * 8 + i] = (g * u) * s;
            }
#pragma unroll
        for (int i = 0; i < 16; i += 2) bf16_round2(o[i], o[i + 1]);
        const int64_t oc0 = col0 / 2;
        if (p.a_next) {
            // two aligned 8-value blocks (oc0 is a multiple of 16), encoded
            // as K2 encodes the f32 values a separate pack would read
#pragma unroll
            for (int h = 0; h < 2; h++) {
                if (oc0 + h * 8 + 8 > p.n_out) break;
                float v[8];
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    v[i] = o[h * 8 + i];
                    bad |= not_finite(v[i]);
                }
                uint8_t enc[9];
                uint32_t bf[4];
                encode_block(v, enc, bf);
                *reinterpret_cast<uint4 *>(p.a_next + row * p.lda_next + oc0 + h * 8) =
                    make_uint4(bf[0], bf[1], bf[2], bf[3]);
            }
        }
        if (!p.c) return bad;
        float *dst = p.c + row * p.ldc + oc0;
        if (oc0 + 16 <= p.n_out && (p.ldc % 4) == 0) {
#pragma unroll
            for (int i = 0; i < 16; i += 4) {
                *reinterpret_cast<float4 *>(dst + i) = make_float4(o[i], o[i + 1], o[i + 2], o[i + 3]);
                bad |= not_finite(o[i]) | not_finite(o[i + 1]) | not_finite(o[i + 2]) | not_finite(o[i + 3]);
            }
        } else {
#pragma unroll
            for (int i = 0; i < 16; i++)
                if (oc0 + i < p.n_out) {
                    dst[i] = o[i];
                    bad |= not_finite(o[i]);
                }
        }
        return bad;
    }
    float o[32];
#pragma unroll
    for (int i = 0; i < 32; i++) o[i] = __uint_as_float(r[i]);
    if (p.mode == MODE_BF16)
#pragma unroll
        for (int i = 0; i < 32; i += 2) bf16_round2(o[i], o[i + 1]);
    if (p.resid) add_residual(p, o, row, col0);
    if (p.c_mc) {
        // a tensor-parallel partial product: summed into every rank's copy
        float *dst = p.c_mc + row * p.ldc + col0;
        if (col0 + 32 <= p.n_out && (p.ldc % 4) == 0 && ((uintptr_t) dst & 15) == 0) {
            bad |= any_not_finite(o);
#pragma unroll
            for (int i = 0; i < 32; i += 4) {
                if (p.mc_store) multimem_st_v4(dst + i, o[i], o[i + 1], o[i + 2], o[i + 3]);
                else multimem_red_add_v4(dst + i, o[i], o[i + 1], o[i + 2], o[i + 3]);
            }
        } else {
#pragma unroll
            for (int i = 0; i < 32; i++)
                if (col0 + i < p.n_out) {
                    if (p.mc_store) multimem_st(dst + i, o[i]);
                    else multimem_red_add(dst + i, o[i]);
                    bad |= not_finite(o[i]);
                }
        }
        return bad;
    }
    float *dst = p.c + row * p.ldc + col0;
    if (col0 + 32 <= p.n_out && (p.ldc % 4) == 0 && ((uintptr_t) dst & 15) == 0) {
        bad |= any_not_finite(o);
#pragma unroll
        for (int i = 0; i < 32; i += 4)
            *reinterpret_cast<float4 *>(dst + i) = make_float4(o[i], o[i + 1], o[i + 2], o[i + 3]);
    } else {
#pragma unroll
        for (int i = 0; i < 32; i++)
            if (col0 + i < p.n_out) {
                dst[i] = o[i];
                bad |= not_finite(o[i]);
            }
    }
    return bad;
}

__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_bf16_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const gemm_params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(((uintptr_t) smem_raw + 1023) & ~(uintptr_t) 1023);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + STAGES * STAGE_BYTES);
    uint64_t *full = bars, *empty = bars + STAGES, *tfull = bars + 2 * STAGES, *tempty = tfull + 2,
             *drain = tempty + 2;
    uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + NUM_BARRIERS);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_holder + 1);

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; a++) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], 4);  // one arrive per epilogue warp
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tmA);
        prefetch_tmap(&tmB);
    }
    if (warp == 1) {
        tmem_alloc(tmem_holder, TMEM_COLS);
        tmem_relinquish();
        tc_fence_before();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_holder;
    const int total = p.num_m * p.num_n;

    auto fail = [&]() {
        *abort_flag = 1;
        atomicOr(p.err, ERR_TIMEOUT);
    };

    if (warp == 0) {
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            uint32_t armed = 0, armed_phase = 0;  // per-stage bits: loads issued, and their phase
            bool ok = true;
            for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
                int mb, nb;
                tile_coords(t, p.num_m, p.num_n, mb, nb);
                for (int kb = 0; kb < p.num_k; kb++) {
                    if (!mbar_wait_bounded(&empty[stage], phase ^ 1, abort_flag, WAIT_LIMIT_NS)) {
                        fail();
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
                    uint8_t *sa = smem + stage * STAGE_BYTES;
                    tma_load_2d(sa, &tmA, &full[stage], kb * BK, mb * BM);
                    tma_load_2d(sa + A_BYTES, &tmB, &full[stage], kb * BK, nb * BN);
                    armed |= 1u << stage;
                    armed_phase = (armed_phase & ~(1u << stage)) | (phase << stage);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            // no copy of ours may land after the block exits
            for (int s = 0; s < STAGES; s++)
                if ((armed & (1u << s)) && !mbar_wait_bounded(&full[s], (armed_phase >> s) & 1u, nullptr, WAIT_LIMIT_NS))
                    fail();
        }
    } else if (warp == 1) {
        if (lane == 0) {
            int stage = 0, acc = 0;
            uint32_t phase = 0, acc_phase = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
                if (!mbar_wait_bounded(&tempty[acc], acc_phase ^ 1, abort_flag, WAIT_LIMIT_NS)) {
                    fail();
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem_base + (uint32_t) (acc * ACC_COLS);
                for (int kb = 0; kb < p.num_k; kb++) {
                    if (!mbar_wait_bounded(&full[stage], phase, abort_flag, WAIT_LIMIT_NS)) {
                        fail();
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint8_t *sa = smem + stage * STAGE_BYTES;
                    const uint64_t adesc = sw128_desc(sa), bdesc = sw128_desc(sa + A_BYTES);
#pragma unroll
                    for (int k = 0; k < BK / 16; k++)
                        tc_mma_bf16(d, adesc + 2 * k, bdesc + 2 * k, IDESC, (kb | k) != 0 ? 1u : 0u);
                    tc_commit(&empty[stage]);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                if (!ok) break;
                tc_commit(&tfull[acc]);
                if (++acc == 2) {
                    acc = 0;
                    acc_phase ^= 1;
                }
            }
            // every MMA we issued is complete before TMEM is freed
            tc_commit(drain);
            if (!mbar_wait_bounded(drain, 0, nullptr, WAIT_LIMIT_NS)) fail();
        }
    } else {
        const int q = warp % 4;  // TMEM lane quarter this warp may read
        int acc = 0;
        uint32_t acc_phase = 0;
        uint32_t bad = 0;
        for (int t = blockIdx.x; t < total; t += gridDim.x) {
            int mb, nb;
            tile_coords(t, p.num_m, p.num_n, mb, nb);
            if (!mbar_wait_bounded(&tfull[acc], acc_phase, abort_flag, WAIT_LIMIT_NS)) {
                fail();
                break;
            }
            tc_fence_after();
            const int64_t row = (int64_t) mb * BM + q * 32 + lane;
            const uint32_t tbase = tmem_base + ((uint32_t) (q * 32) << 16) + (uint32_t) (acc * ACC_COLS);
            uint32_t r[32];
            for (int ch = 0; ch < BN / 32; ch++) {
                tmem_ld_32x32b_x32(tbase + (uint32_t) (ch * 32), r);
                tmem_ld_wait();
                if (ch == BN / 32 - 1) {
                    // the warp's loads of this accumulator are done: one
                    // elected arrive hands it back to the MMA warp
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&tempty[acc]);
                }
                const int64_t col0 = (int64_t) nb * BN + ch * 32;
                if (col0 < p.N) bad |= store_chunk(p, r, row, col0);
            }
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1;
            }
        }
        if (p.c_mc) asm volatile("fence.acq_rel.sys;" ::: "memory");  // the reductions are performed before we exit
        if (__any_sync(0xffffffffu, bad) && lane == 0) atomicOr(p.err, ERR_NOT_FINITE);
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

// ---------------------------------------------------------------------------
// The CTA-pair kernel: a cluster of 2 CTAs on one TPC computes a 256x256
// tile with tcgen05.mma.cta_group::2 (M=256 across the pair, N=256). Each CTA
// loads only its 128 rows of A and its 128 rows (half) of B, so per SM every
// 64-deep k step moves 32 KB into shared memory instead of 48 KB for the same
// 128x256 of output, and the pair leader issues one MMA for both SMs.
//
// Barriers (same offsets in both CTAs):
//   full[s]    leader: armed by the leader's producer with both CTAs' bytes;
//              both CTAs' TMA loads complete on it
//   empty[s]   each CTA: the leader's commit, multicast to both
//   tfull[a]   each CTA: the leader's commit, multicast to both
//   tempty[a]  leader: each of the pair's 8 epilogue warps arrives once
// Cluster syncs bracket barrier set-up and TMEM release, so neither CTA's
// barriers are used before they exist or after it exits.
// ---------------------------------------------------------------------------

constexpr int P_BM = 256;

// The pair kernel's shape for an N tile of P_BN columns (a multiple of 32,
// at most 256): each CTA holds 128 rows of A and P_BN/2 rows of B per stage;
// each of the 4 epilogue warps has NBUF 32 x 32 fp32 staging buffers for its
// TMA stores; the ring takes what is left of 224 KB. The two accumulators
// sit 256 TMEM columns apart.
template <int BN_T, int NBUF>
struct pair_cfg {
    static constexpr int P_BN = BN_T;
    static constexpr int P_EPI_BYTES = 4 * NBUF * 32 * 32 * 4;
    static constexpr int P_A_BYTES = 128 * BK * 2;       // this CTA's half of A
    static constexpr int P_B_BYTES = (BN_T / 2) * BK * 2; // this CTA's half of B
    static constexpr int P_STAGE_BYTES = P_A_BYTES + P_B_BYTES;
    static constexpr int P_STAGES = (229376 - P_EPI_BYTES) / P_STAGE_BYTES;
    static constexpr int P_NUM_BARRIERS = 2 * P_STAGES + 5;
    static constexpr int P_SMEM_BYTES = 1024 + P_STAGES * P_STAGE_BYTES + P_EPI_BYTES + P_NUM_BARRIERS * 8 + 16;
    static constexpr uint32_t P_IDESC = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t) (BN_T >> 3) << 17) |
                                        ((uint32_t) (P_BM >> 4) << 24);
    static_assert(BN_T % 32 == 0 && BN_T <= 256 && P_STAGE_BYTES % 1024 == 0, "pair tile shape");
    static_assert(NBUF >= 2 && P_STAGES >= 4, "staging buffers and ring stages");
};

// A grouped launch: up to MAX_SEG weights sharing one A (q, k and v; gate
// and up), each with its own B, output and mode. Their N tiles are laid end
// to end, so one persistent launch runs them all and no kernel tail
// separates them (the reference submits such a group as one NPU runlist,
// src/xdna-npu.cpp:476-531).
constexpr int MAX_SEG = 4;

// Up to MAX_PEERS other GPUs' copies of each output, stored into by the
// epilogue's TMA beside the local one (an N-shard's all-gather).
constexpr int MAX_PEERS = 7;

struct pair_maps {
    CUtensorMap b[MAX_SEG], c[MAX_SEG];
    CUtensorMap peer[MAX_SEG][MAX_PEERS];
    CUtensorMap c16[MAX_SEG][MAX_PEERS + 1];  // bf16 copies: 32 x 32 boxes, 64-byte swizzle
};

struct pair_params {
    gemm_params seg[MAX_SEG];  // per weight: N, n_out, ldc, c, mode, tma_store (M, K, err shared)
    int tile0[MAX_SEG + 1];    // first N tile of each segment; tile0[nseg] = all N tiles
    int nseg, num_m, num_n, num_k;
    int raster;                // RASTER_*
    int stream_hint;           // the streamed operand's loads carry an evict-first L2 hint
    // stream-K: tiles [0, dp_tiles) run whole, one per pair per wave; the
    // sk_tiles after them are cut into runs of sk_q k-blocks, pair p taking
    // [p * sk_q, (p + 1) * sk_q) of their (tile, k-block) space
    int dp_tiles, sk_tiles;
    int64_t sk_q;
    int sk_epoch;  // this launch's flag value: stale flags of an abandoned launch never match
    int64_t M;
    unsigned *err;
};

// Stream-K partial sums: a CTA whose last run stops inside a tile leaves its
// 128 rows x (at most) 256 fp32 columns here, in its own slot, and raises its
// flag; the CTA that finishes the tile adds them in k order and clears the
// flags. One workspace per device: launches that may use it are serialised
// across streams by the launcher.
constexpr int SK_SLOTS = 160;
constexpr int SK_SLOT_FLOATS = 128 * 256;
// A CTA's partial tile in the workspace, in the order the epilogue holds it:
// warp q, 32-column chunk ch, 4-column group g, then the warp's 32 lanes (one
// row each), four floats apiece. Each float4 access of a warp is then 512
// contiguous bytes; the writer and the reader of a slot share (q, lane) for
// every row, as both are the same rank of their pair.
__device__ __forceinline__ size_t sk_off(int q, int ch, int g, int lane) {
    return ((size_t) ((q * 8 + ch) * 8 + g) * 32 + lane) * 4;
}
__device__ float g_sk_part[SK_SLOTS * SK_SLOT_FLOATS];
__device__ int g_sk_flag[SK_SLOTS];

// The runs of one pair. Its stretch of the stream-K space is walked one
// (tile, k-block range) at a time from the END back to its start, so the
// run that stops inside a tile (whose partial sum another pair waits for)
// comes before the run that finishes a tile started by the pair before it:
// no pair waits on a pair that is itself waiting. That first stream-K run
// goes ahead of the pair's whole tiles, so every partial is published at the
// start of the launch and a short run never follows a whole tile directly
// (the MMAs of the run after it would wait for that tile's epilogue to free
// its accumulator).
struct unit_iter {
    int i = 0;
    bool lead = true;        // the stretch's first run is still to come, ahead of the whole tiles
    int64_t u0 = 0, u1 = 0;  // the stretch still to walk, [u0, u1)
    __device__ unit_iter(const pair_params &pp, int pair) {
        const int64_t end = (int64_t) pp.sk_tiles * pp.num_k;
        u0 = (int64_t) pair * pp.sk_q;
        u1 = u0 + pp.sk_q < end ? u0 + pp.sk_q : end;
        if (u0 > u1) u0 = u1;
    }
    __device__ bool next(const pair_params &pp, int pair, int npairs, int &t, int &kb0, int &kb1) {
        if (lead) {
            lead = false;
            if (u1 > u0) return take(pp, t, kb0, kb1);
        }
        const int td = pair + i * npairs;
        if (td < pp.dp_tiles) {
            i++;
            t = td;
            kb0 = 0;
            kb1 = pp.num_k;
            return true;
        }
        if (u1 <= u0) return false;
        return take(pp, t, kb0, kb1);
    }
    // the last (tile, k-block range) of what is left of the stretch
    __device__ bool take(const pair_params &pp, int &t, int &kb0, int &kb1) {
        const int64_t st = (u1 - 1) / pp.num_k, ts = st * pp.num_k;
        const int64_t start = u0 > ts ? u0 : ts;
        t = pp.dp_tiles + (int) st;
        kb0 = (int) (start - ts);
        kb1 = (int) (u1 - ts);
        u1 = start;
        return true;
    }
};

// The order the persistent pairs walk the tiles in. Pair p takes tiles p,
// p + pairs, ..., so each wave is a run of consecutive tiles; the order is
// chosen per launch so the operand every wave re-reads stays in L2:
//   RASTER_ROWS    an M block's N tiles together: A streamed once, B (small
//                  N x K) read from L2 by every wave
//   RASTER_COLS    an N tile's M blocks together: B streamed once, A (small
//                  M x K) read from L2
//   RASTER_GROUPS  GROUP_M M blocks at a time, their N tiles within: when
//                  neither operand fits
enum { RASTER_GROUPS = 0, RASTER_ROWS = 1, RASTER_COLS = 2 };

__device__ __forceinline__ void pair_tile_coords(int t, const pair_params &pp, int &mb, int &nb) {
    if (pp.raster == RASTER_ROWS) {
        mb = t / pp.num_n;
        nb = t % pp.num_n;
    } else if (pp.raster == RASTER_COLS) {
        nb = t / pp.num_m;
        mb = t % pp.num_m;
    } else {
        tile_coords(t, pp.num_m, pp.num_n, mb, nb);
    }
}

// SK: whether this instance walks stream-K runs (a separate instance, so the
// whole-tile kernel carries none of that code or its registers).
template <int BN_T, bool SK, int NBUF>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_bf16_tc_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ pair_maps maps,
                             const __grid_constant__ pair_params pp) {
    using C = pair_cfg<BN_T, NBUF>;
    constexpr int P_BN = C::P_BN, P_A_BYTES = C::P_A_BYTES, P_STAGE_BYTES = C::P_STAGE_BYTES,
                  P_STAGES = C::P_STAGES, P_NUM_BARRIERS = C::P_NUM_BARRIERS, P_EPI_BYTES = C::P_EPI_BYTES;
    constexpr uint32_t P_IDESC = C::P_IDESC;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(((uintptr_t) smem_raw + 1023) & ~(uintptr_t) 1023);
    uint8_t *epi = smem + P_STAGES * P_STAGE_BYTES;  // 1 KB aligned
    uint64_t *bars = reinterpret_cast<uint64_t *>(epi + P_EPI_BYTES);
    uint64_t *full = bars, *empty = bars + P_STAGES, *tfull = bars + 2 * P_STAGES, *tempty = tfull + 2,
             *drain = tempty + 2;
    uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + P_NUM_BARRIERS);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_holder + 1);

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    if (threadIdx.x == 0) {
        for (int s = 0; s < P_STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; a++) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], 8);  // one arrive per epilogue warp of the pair
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tmA);
        for (int s = 0; s < pp.nseg; s++) prefetch_tmap(&maps.b[s]);
    }
    if (warp == 1) {
        tmem_alloc_pair(tmem_holder, TMEM_COLS);
        tmem_relinquish_pair();
        tc_fence_before();
    }
    cluster_sync();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_holder;
    const int pair = blockIdx.x / 2, npairs = gridDim.x / 2;

    // global N tile -> (segment, its own N tile)
    auto locate = [&](int nbg, int &seg, int &nb) {
        seg = 0;
        while (seg + 1 < pp.nseg && nbg >= pp.tile0[seg + 1]) seg++;
        nb = nbg - pp.tile0[seg];
    };
    auto fail = [&]() {
        *abort_flag = 1;
        atomicOr(pp.err, ERR_TIMEOUT);
    };

    if (warp == 0) {
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            uint32_t armed = 0, armed_phase = 0;
            bool ok = true;
            const uint64_t pol = l2_evict_first_policy();
            const bool hint_a = pp.stream_hint && pp.raster == RASTER_ROWS;
            const bool hint_b = pp.stream_hint && pp.raster != RASTER_ROWS;
            unit_iter it(pp, pair);
            int t, kb0, kb1;
            while (ok && it.next(pp, pair, npairs, t, kb0, kb1)) {
                int mb, nbg, seg, nb;
                pair_tile_coords(t, pp, mb, nbg);
                locate(nbg, seg, nb);
                for (int kb = kb0; kb < kb1; kb++) {
                    if (!mbar_wait_bounded(&empty[stage], phase ^ 1, abort_flag, WAIT_LIMIT_NS)) {
                        fail();
                        ok = false;
                        break;
                    }
                    if (leader) mbar_arrive_expect_tx(&full[stage], 2 * P_STAGE_BYTES);
                    const uint32_t bar = map_to_rank(&full[stage], 0);
                    uint8_t *sa = smem + stage * P_STAGE_BYTES;
                    // the operand this raster streams is read once: evict-first
                    if (hint_a)
                        tma_load_2d_pair_hint(sa, &tmA, bar, kb * BK, mb * P_BM + (int) rank * 128, pol);
                    else
                        tma_load_2d_pair(sa, &tmA, bar, kb * BK, mb * P_BM + (int) rank * 128);
                    if (hint_b)
                        tma_load_2d_pair_hint(sa + P_A_BYTES, &maps.b[seg], bar, kb * BK,
                                              nb * P_BN + (int) rank * (P_BN / 2), pol);
                    else
                        tma_load_2d_pair(sa + P_A_BYTES, &maps.b[seg], bar, kb * BK, nb * P_BN + (int) rank * (P_BN / 2));
                    armed |= 1u << stage;
                    armed_phase = (armed_phase & ~(1u << stage)) | (phase << stage);
                    if (++stage == P_STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            // our copies have all landed before the pair tears down: the
            // leader sees them complete on its full barriers, the peer waits
            // for the leader's MMAs (which consumed them) through empty
            for (int s = 0; s < P_STAGES; s++) {
                if (!(armed & (1u << s))) continue;
                const bool done = leader ? mbar_wait_bounded(&full[s], (armed_phase >> s) & 1u, nullptr, WAIT_LIMIT_NS)
                                         : mbar_wait_bounded(&empty[s], (armed_phase >> s) & 1u, nullptr, WAIT_LIMIT_NS);
                if (!done) fail();
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && leader) {
            int stage = 0, acc = 0;
            uint32_t phase = 0, acc_phase = 0;
            bool ok = true;
            unit_iter it(pp, pair);
            int t, kb0, kb1;
            while (ok && it.next(pp, pair, npairs, t, kb0, kb1)) {
                if (!mbar_wait_bounded(&tempty[acc], acc_phase ^ 1, abort_flag, WAIT_LIMIT_NS)) {
                    fail();
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem_base + (uint32_t) (acc * ACC_COLS);
                for (int kb = kb0; kb < kb1; kb++) {
                    if (!mbar_wait_bounded(&full[stage], phase, abort_flag, WAIT_LIMIT_NS)) {
                        fail();
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint8_t *sa = smem + stage * P_STAGE_BYTES;
                    const uint64_t adesc = sw128_desc(sa), bdesc = sw128_desc(sa + P_A_BYTES);
#pragma unroll
                    for (int k = 0; k < BK / 16; k++)
                        tc_mma_bf16_pair(d, adesc + 2 * k, bdesc + 2 * k, P_IDESC, (kb != kb0 || k != 0) ? 1u : 0u);
                    tc_commit_pair_mc(&empty[stage], 0x3);
                    if (++stage == P_STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                if (!ok) break;
                tc_commit_pair_mc(&tfull[acc], 0x3);
                if (++acc == 2) {
                    acc = 0;
                    acc_phase ^= 1;
                }
            }
            tc_commit_pair(map_to_rank(drain, 0));
            if (!mbar_wait_bounded(drain, 0, nullptr, WAIT_LIMIT_NS)) fail();
        }
    } else {
        const int q = warp % 4;
        const uint32_t tempty_leader0 = map_to_rank(&tempty[0], 0), tempty_leader1 = map_to_rank(&tempty[1], 0);
        int acc = 0;
        uint32_t acc_phase = 0;
        uint32_t bad = 0;
        bool stored = false;
        const uint64_t out_pol = l2_evict_first_policy();  // outputs are written once
        unit_iter it(pp, pair);
        int t, kb0, kb1;
        bool dead = false;
        while (it.next(pp, pair, npairs, t, kb0, kb1)) {
            int mb, nbg, seg, nb;
            pair_tile_coords(t, pp, mb, nbg);
            locate(nbg, seg, nb);
            const gemm_params &p = pp.seg[seg];
            if (p.resid) {
                // bring this row's residual into L2 while the tile's MMAs run
                const int64_t prow = (int64_t) mb * P_BM + rank * 128 + q * 32 + lane;
                const int64_t pc0 = (int64_t) nb * P_BN;
                if (prow < p.M)
                    for (int c = 0; c < P_BN && pc0 + c < p.n_out; c += 32)
                        asm volatile("prefetch.global.L2 [%0];" ::"l"(p.resid + prow * p.ldr + pc0 + c));
            }
            if (!mbar_wait_bounded(&tfull[acc], acc_phase, abort_flag, WAIT_LIMIT_NS)) {
                fail();
                break;
            }
            tc_fence_after();
            // stream-K: this run stops inside the tile (its sum goes to the
            // workspace), or finishes a tile that earlier runs started
            const bool part = SK && kb1 < pp.num_k, fin = SK && !part && kb0 > 0;
            const int j0 = fin ? (int) ((int64_t) (t - pp.dp_tiles) * pp.num_k / pp.sk_q) : 0;
            if (fin && !dead)
                for (int j = j0; j < pair; j++)
                    if (!flag_wait_bounded(&g_sk_flag[2 * j + rank], pp.sk_epoch, abort_flag, WAIT_LIMIT_NS)) {
                        fail();
                        dead = true;  // keep step with the other warps through the barriers below
                        break;
                    }
            const int64_t row0 = (int64_t) mb * P_BM + rank * 128 + q * 32, row = row0 + lane;
            const uint32_t tbase = tmem_base + ((uint32_t) (q * 32) << 16) + (uint32_t) (acc * ACC_COLS);
            // each chunk's TMEM load goes out while the chunk before it is
            // stored, so its latency overlaps that work
            uint32_t r[32], nx[32];
            tmem_ld_32x32b_x32(tbase, nx);
            for (int ch = 0; ch < P_BN / 32; ch++) {
                // the residual's loads (or, finishing a stream-K tile, the
                // first partial's) go out before the wait for this chunk
                float4 rr[8];
                const int64_t rcol0 = (int64_t) nb * P_BN + ch * 32;
                const bool rfast = p.resid && p.tma_store && row < p.M && rcol0 + 32 <= p.n_out &&
                                   (p.ldr % 4) == 0 && ((uintptr_t) p.resid & 15) == 0;
                const bool sum_in = fin && !dead;
                if (sum_in) {
                    const float *src = g_sk_part + (size_t) (2 * j0 + rank) * SK_SLOT_FLOATS;
#pragma unroll
                    for (int g = 0; g < 8; g++) rr[g] = *reinterpret_cast<const float4 *>(src + sk_off(q, ch, g, lane));
                } else if (rfast) {
                    const float4 *src = reinterpret_cast<const float4 *>(p.resid + row * p.ldr + rcol0);
#pragma unroll
                    for (int i = 0; i < 8; i++) rr[i] = src[i];
                }
                tmem_ld_wait(nx);
#pragma unroll
                for (int i = 0; i < 32; i++) r[i] = nx[i];
                if (ch + 1 < P_BN / 32) tmem_ld_32x32b_x32(tbase + (uint32_t) ((ch + 1) * 32), nx);
                if (ch == P_BN / 32 - 1) {
                    // the warp's loads of this accumulator are done: one
                    // elected arrive per warp (8 for the pair, not 256
                    // arrivals of which half cross to the leader CTA) hands
                    // it back to the MMA warp
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive_cluster(acc ? tempty_leader1 : tempty_leader0);
                }
                if (part) {
                    float *dst = g_sk_part + (size_t) blockIdx.x * SK_SLOT_FLOATS;
#pragma unroll
                    for (int g = 0; g < 8; g++)
                        *reinterpret_cast<float4 *>(dst + sk_off(q, ch, g, lane)) = make_float4(
                            __uint_as_float(r[4 * g]), __uint_as_float(r[4 * g + 1]), __uint_as_float(r[4 * g + 2]),
                            __uint_as_float(r[4 * g + 3]));
                    continue;
                }
                if (sum_in) {
                    for (int j = j0; j < pair; j++) {
                        if (j > j0) {
                            const float *src = g_sk_part + (size_t) (2 * j + rank) * SK_SLOT_FLOATS;
#pragma unroll
                            for (int g = 0; g < 8; g++)
                                rr[g] = *reinterpret_cast<const float4 *>(src + sk_off(q, ch, g, lane));
                        }
#pragma unroll
                        for (int g = 0; g < 8; g++) {
                            r[4 * g] = __float_as_uint(__uint_as_float(r[4 * g]) + rr[g].x);
                            r[4 * g + 1] = __float_as_uint(__uint_as_float(r[4 * g + 1]) + rr[g].y);
                            r[4 * g + 2] = __float_as_uint(__uint_as_float(r[4 * g + 2]) + rr[g].z);
                            r[4 * g + 3] = __float_as_uint(__uint_as_float(r[4 * g + 3]) + rr[g].w);
                        }
                    }
                    if (rfast) {
                        // the residual after the partials (it is in L2: prefetched at the tile's start)
                        const float4 *src = reinterpret_cast<const float4 *>(p.resid + row * p.ldr + rcol0);
#pragma unroll
                        for (int i = 0; i < 8; i++) rr[i] = src[i];
                    }
                }
                const int64_t col0 = (int64_t) nb * P_BN + ch * 32;
                if (col0 >= p.N) continue;
                if (!p.tma_store && !p.c_mc && !p.n_c16) {
                    bad |= store_chunk(p, r, row, col0);
                    continue;
                }
                if (p.n_c16) {
                    // the chunk in bf16 (bf16 mode: the rounded values are
                    // bf16 exactly): 32 rows x 64 bytes, 64-byte swizzle,
                    // TMA-stored into every copy
                    uint8_t *buf = epi + (q * NBUF + (ch % NBUF)) * 4096;
                    if (lane == 0) bulk_wait_read<NBUF - 1>();  // the store NBUF chunks ago has read this buffer
                    __syncwarp();
                    float o[32];
#pragma unroll
                    for (int i = 0; i < 32; i++) o[i] = __uint_as_float(r[i]);
#pragma unroll
                    for (int i = 0; i < 32; i += 2) bf16_round2(o[i], o[i + 1]);
                    bad |= any_not_finite(o);
#pragma unroll
                    for (int u = 0; u < 4; u++) {
                        uint32_t w[4];
#pragma unroll
                        for (int k = 0; k < 4; k++)
                            w[k] = __byte_perm(__float_as_uint(o[8 * u + 2 * k]), __float_as_uint(o[8 * u + 2 * k + 1]),
                                               0x7632);
                        *reinterpret_cast<uint4 *>(buf + lane * 64 + ((u ^ ((lane >> 1) & 3)) << 4)) =
                            make_uint4(w[0], w[1], w[2], w[3]);
                    }
                    fence_proxy_async_shared();
                    __syncwarp();
                    if (lane == 0) {
                        for (int r2 = 0; r2 < p.n_c16; r2++)
                            tma_store_2d_hint(&maps.c16[seg][r2], buf, (int32_t) col0, (int32_t) row0, out_pol);
                        bulk_commit_group();
                        stored = true;
                    }
                    continue;
                }
                // this warp's 32 rows x 32 columns through a 128-byte-swizzled
                // staging buffer (NBUF of them in turn) and one TMA store
                uint8_t *buf = epi + (q * NBUF + (ch % NBUF)) * 4096;
                if (lane == 0) bulk_wait_read<NBUF - 1>();  // the store NBUF chunks ago has read this buffer
                __syncwarp();
                float o[32];
#pragma unroll
                for (int i = 0; i < 32; i++) o[i] = __uint_as_float(r[i]);
                if (p.mode == MODE_BF16)
#pragma unroll
                    for (int i = 0; i < 32; i += 2) bf16_round2(o[i], o[i + 1]);
                if (rfast) {
#pragma unroll
                    for (int i = 0; i < 8; i++) {
                        o[4 * i] = __fadd_rn(rr[i].x, o[4 * i]);
                        o[4 * i + 1] = __fadd_rn(rr[i].y, o[4 * i + 1]);
                        o[4 * i + 2] = __fadd_rn(rr[i].z, o[4 * i + 2]);
                        o[4 * i + 3] = __fadd_rn(rr[i].w, o[4 * i + 3]);
                    }
                } else if (p.resid && row < p.M) {
                    add_residual(p, o, row, col0);
                }
                // rows past M and columns past the output hold the operands' zero
                // fill (TMA's out-of-bounds fill, the weights' zero padding rows),
                // so the whole chunk can be checked without a branch
                bad |= any_not_finite(o);
#pragma unroll
                for (int j = 0; j < 8; j++)
                    *reinterpret_cast<float4 *>(buf + lane * 128 + ((j ^ (lane & 7)) << 4)) =
                        make_float4(o[4 * j], o[4 * j + 1], o[4 * j + 2], o[4 * j + 3]);
                if (p.c_mc) {
                    // a tensor-parallel partial: read the staged 32 x 32 back by
                    // rows (8 lanes a row, 4 rows an instruction) and add each
                    // 512-byte run into every rank's copy through the NVSwitch
                    __syncwarp();
#pragma unroll
                    for (int it = 0; it < 8; it++) {
                        const int rl = it * 4 + lane / 8, u = lane % 8;
                        const float4 v = *reinterpret_cast<const float4 *>(buf + rl * 128 + ((u ^ (rl & 7)) << 4));
                        const int64_t grow = row0 + rl, gcol = col0 + u * 4;
                        if (grow < p.M) {
                            float *dst = p.c_mc + grow * p.ldc + gcol;
                            if (gcol + 4 <= p.n_out && ((uintptr_t) dst & 15) == 0) {
                                if (p.mc_store) multimem_st_v4(dst, v.x, v.y, v.z, v.w);
                                else multimem_red_add_v4(dst, v.x, v.y, v.z, v.w);
                            } else {
                                const float e[4] = { v.x, v.y, v.z, v.w };
                                for (int i = 0; i < 4; i++)
                                    if (gcol + i < p.n_out) {
                                        if (p.mc_store) multimem_st(dst + i, e[i]);
                                        else multimem_red_add(dst + i, e[i]);
                                    }
                            }
                        }
                    }
                    __syncwarp();
                    continue;
                }
                fence_proxy_async_shared();
                __syncwarp();
                if (lane == 0) {
                    tma_store_2d_hint(&maps.c[seg], buf, (int32_t) col0, (int32_t) row0, out_pol);
                    for (int r = 0; r < p.n_peers; r++)
                        tma_store_2d_hint(&maps.peer[seg][r], buf, (int32_t) col0, (int32_t) row0, out_pol);
                    bulk_commit_group();
                    stored = true;
                }
            }
            if (part || fin) {
                // the four epilogue warps are through this tile: publish our
                // partial, or free the partials we consumed for the next launch
                named_barrier(1, 128);
                if (q == 0 && lane == 0) {
                    if (part) {
                        __threadfence();
                        flag_release(&g_sk_flag[blockIdx.x], pp.sk_epoch);
                    } else {
                        for (int j = j0; j < pair; j++) g_sk_flag[2 * j + rank] = 0;
                    }
                }
            }
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1;
            }
        }
        if (stored) bulk_wait_all();  // every store has landed before the block exits
        bool mc = false;
        for (int sg = 0; sg < pp.nseg; sg++)
            mc = mc || pp.seg[sg].c_mc != nullptr || pp.seg[sg].n_peers > 0 || pp.seg[sg].n_c16 > 0;
        if (mc) fence_proxy_async_global();  // the peers' copies: TMA's writes ordered before the fence below
        if (mc) asm volatile("fence.acq_rel.sys;" ::: "memory");  // the reductions are performed before we exit
        if (__any_sync(0xffffffffu, bad) && lane == 0) atomicOr(pp.err, ERR_NOT_FINITE);
    }

    tc_fence_before();
    __syncthreads();
    cluster_sync();  // no barrier of either CTA is signalled after this
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, TMEM_COLS);
    }
}

PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

// A row-major bf16 matrix [rows][ld] as 64 x box_rows tiles, 128-byte swizzle.
bool make_tmap(CUtensorMap *m, const void *base, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
    auto fn = get_encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = { (cuuint64_t) cols, (cuuint64_t) rows };
    cuuint64_t strides[1] = { (cuuint64_t) ld * 2 };
    cuuint32_t box[2] = { (cuuint32_t) BK, (cuuint32_t) box_rows };
    cuuint32_t estr[2] = { 1, 1 };
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The f32 output [rows][ld] as 32 x 32 tiles, 128-byte swizzle, for the
// epilogue's TMA stores.
bool make_tmap_out(CUtensorMap *m, void *base, int64_t rows, int64_t cols, int64_t ld) {
    auto fn = get_encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = { (cuuint64_t) cols, (cuuint64_t) rows };
    cuuint64_t strides[1] = { (cuuint64_t) ld * 4 };
    cuuint32_t box[2] = { 32, 32 };
    cuuint32_t estr[2] = { 1, 1 };
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
           CUDA_SUCCESS;
}

// A bf16 output [rows][ld] as 32 x 32 tiles, 64-byte swizzle, for the
// epilogue's bf16 copies.
bool make_tmap_out16(CUtensorMap *m, void *base, int64_t rows, int64_t cols, int64_t ld) {
    auto fn = get_encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = { (cuuint64_t) cols, (cuuint64_t) rows };
    cuuint64_t strides[1] = { (cuuint64_t) ld * 2 };
    cuuint32_t box[2] = { 32, 32 };
    cuuint32_t estr[2] = { 1, 1 };
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
           CUDA_SUCCESS;
}

// The SMs the persistent GEMM spreads over: all of them, or at most
// ZEST_GEMM_MAX_SMS (even), leaving the rest to kernels that must run beside
// it, such as a collective overlapping the next row chunk's GEMMs.
int num_sms() {
    static int sms = 0;
    if (!sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (sms <= 0) sms = 148;
        if (const char *cap = getenv("ZEST_GEMM_MAX_SMS")) {
            const int c = atoi(cap) & ~1;
            if (c >= 2 && c < sms) sms = c;
        }
    }
    return sms;
}

// Stream-K plan: when the last wave of whole tiles would leave pairs idle,
// that wave and the full wave before it are cut into equal runs of k-blocks,
// one run per pair. By default only where a quarter or more of the launch's
// pair-slots would sit idle and K is 4096 or more, or K is 8192 or more and
// there is at least one full wave: measured on the configs' shapes (device
// time per launch, whole tiles -> stream-K), C3 o 51 -> 46 us (idle 0.46, 64
// k-blocks), C3 down 104 -> 80 (0.46), C5 M=1024 down 61 -> 54 (0.57), C4
// M=2048 down 327 -> 281 (0.28), C2 down about 330 -> 292 (0.14, 152
// k-blocks, mean of 5 runs); while C1 (0.32 idle but 40 k-blocks) 51 -> 54,
// C5 M=2048 down (one wave of 64 tiles, 0.14 idle) 66 -> 74, and the shorter
// launches with less idle lose 2-10 %: each split tile adds an exposed
// epilogue, and under the power cap the busy pairs of a ragged wave run at
// higher clocks.
// ZEST_GEMM_SK=1 splits whenever the shape allows, ZEST_GEMM_SK=0 never.
bool plan_stream_k(gemm_plan &gp, int pairs) {
    const int64_t tiles = gp.tiles;
    static const int mode = [] {
        const char *s = getenv("ZEST_GEMM_SK");
        return s && s[0] == '1' ? 1 : (s && s[0] == '0' ? 0 : 2);
    }();
    if (mode == 0) return false;
    if (mode == 2) {
        const int64_t slots = (tiles + pairs - 1) / pairs * pairs;
        const bool ragged = gp.num_k >= 64 && 4 * (slots - tiles) >= slots;
        const bool long_k = gp.num_k >= 128 && tiles >= pairs;
        if (!ragged && !long_k) return false;
    }
    const int64_t full = tiles / pairs, rem = tiles % pairs;
    if (rem == 0 || 2 * pairs > SK_SLOTS || rem > (pairs * 7) / 8) return false;
    if (full == 0 && rem < 2) return false;
    const int64_t sk_tiles = rem + (full >= 1 ? pairs : 0);
    const int64_t q = (sk_tiles * gp.num_k + pairs - 1) / pairs;
    if (q < 4) return false;
    gp.dp_tiles = (int) ((full >= 1 ? full - 1 : 0) * pairs);
    gp.sk_tiles = (int) sk_tiles;
    gp.sk_q = q;
    return true;
}

// The stream-K workspace is one per device, so launches that may use it run
// one at a time. A live launch on another stream than the last live one
// waits for it (an event recorded after each). A launch being captured into
// a CUDA graph runs nothing now, so it can neither wait for a live launch
// nor order the ones after it: it leaves the live record alone and takes
// stream-K only when no live launch on another stream may still hold the
// workspace and no other stream of the same capture took it (two branches of
// one graph may run at once). A graph's own stream-K launches are thereby
// ordered within the graph; replaying it beside live launches on other
// streams is the caller's to order.
struct sk_owner {
    cudaStream_t last = nullptr;  // the stream of the last live stream-K launch
    cudaEvent_t done = nullptr;   // recorded on it after that launch
    bool recorded = false;
    unsigned long long cap_id = 0;  // the last capture that took stream-K, and its stream
    cudaStream_t cap_stream = nullptr;
    int epoch = 0;
};
std::mutex g_sk_mu;
sk_owner g_sk_owner[64];

// What a launch on `st` may do with the workspace, given the record `o`:
// run stream-K (true) and, for a live launch, first wait for `o.done`.
// Updates the record for a launch that takes it. Host logic only.
bool sk_decide(sk_owner &o, cudaStream_t st, bool capturing, unsigned long long cap_id, bool *wait) {
    *wait = false;
    if (capturing) {
        if (o.recorded && o.last != st) return false;
        if (o.cap_id == cap_id && o.cap_stream != st) return false;
        o.cap_id = cap_id;
        o.cap_stream = st;
        return true;
    }
    *wait = o.recorded && o.last != st;
    o.last = st;
    return true;
}

bool sk_claim(cudaStream_t st, int *epoch) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev >= 64) return false;
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    unsigned long long cap_id = 0;
    if (cudaStreamGetCaptureInfo(st, &cs, &cap_id) != cudaSuccess) return false;
    const bool capturing = cs != cudaStreamCaptureStatusNone;
    std::lock_guard<std::mutex> lk(g_sk_mu);
    sk_owner &o = g_sk_owner[dev];
    if (!o.done && cudaEventCreateWithFlags(&o.done, cudaEventDisableTiming) != cudaSuccess) return false;
    sk_owner before = o;
    bool wait = false;
    if (!sk_decide(o, st, capturing, cap_id, &wait)) return false;
    if (wait && cudaStreamWaitEvent(st, o.done, 0) != cudaSuccess) {
        o = before;
        return false;
    }
    o.epoch = o.epoch == 0x7fffffff ? 1 : o.epoch + 1;
    *epoch = o.epoch;
    return true;
}

void sk_release(cudaStream_t st) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev >= 64) return;
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    cudaStreamIsCapturing(st, &cs);
    std::lock_guard<std::mutex> lk(g_sk_mu);
    sk_owner &o = g_sk_owner[dev];
    if (cs == cudaStreamCaptureStatusNone) o.recorded = cudaEventRecord(o.done, st) == cudaSuccess;
}

// The pair kernel for an N tile of BN_T over a group of weights sharing A:
// B's tensor maps (BN_T/2-row boxes, one per CTA), the outputs' for TMA
// stores, a cluster-of-2 launch.
template <int BN_T, int NBUF>
int launch_pair_group(const CUtensorMap &ta, int64_t M, int64_t K, int nseg, const gemm_seg *segs, const gemm_plan &gp,
                      unsigned *err_flag, cudaStream_t st) {
    using C = pair_cfg<BN_T, NBUF>;
    pair_maps maps;
    pair_params pp;
    memset(&maps, 0, sizeof maps);
    memset(&pp, 0, sizeof pp);
    pp.nseg = nseg;
    pp.M = M;
    pp.err = err_flag;
    pp.num_m = gp.num_m;
    pp.num_k = gp.num_k;
    int tiles_n = 0;
    for (int s = 0; s < nseg; s++) {
        const gemm_seg &g = segs[s];
        if (!make_tmap(&maps.b[s], g.b, g.N, K, g.ldb, BN_T / 2))
            return set_error("gemm: cannot build the TMA descriptors");
        gemm_params &p = pp.seg[s];
        p.M = M;
        p.N = g.N;
        p.K = K;
        p.ldc = g.ldc;
        p.n_out = g.n_out;
        p.c = g.c;
        p.err = err_flag;
        p.mode = g.mode;
        p.resid = g.resid;
        p.ldr = g.ldr;
        p.a_next = g.a_next;
        p.lda_next = g.lda_next;
        p.c_mc = g.c_mc;
        p.mc_store = g.mc_store;
        // TMA stores need 16-byte aligned rows; SwiGLU halves the width and keeps direct stores
        p.tma_store = g.mode != MODE_SWIGLU && g.c && g.ldc % 4 == 0 && ((uintptr_t) g.c & 15) == 0 &&
                      make_tmap_out(&maps.c[s], g.c, M, g.n_out, g.ldc);
        p.n_peers = 0;
        if (g.n_peers > 0) {
            if (!p.tma_store || g.n_peers > MAX_PEERS || !g.c_peers)
                return set_error("gemm: peer copies need a TMA-stored output (fp32 or bf16, 16-byte aligned rows) "
                                 "and at most 7 peers");
            for (int r = 0; r < g.n_peers; r++)
                if (!g.c_peers[r] || ((uintptr_t) g.c_peers[r] & 15) ||
                    !make_tmap_out(&maps.peer[s][r], g.c_peers[r], M, g.n_out, g.ldc))
                    return set_error("gemm: cannot build the TMA descriptor of a peer's copy");
            p.n_peers = g.n_peers;
        }
        p.n_c16 = 0;
        if (g.n_c16 > 0) {
            if (g.mode != MODE_BF16 || g.c || g.c_mc || g.resid || g.n_peers || g.n_c16 > MAX_PEERS + 1 || !g.c16 ||
                g.ldc16 < g.n_out || g.ldc16 % 8)
                return set_error("gemm: bf16 copies take a bf16-mode output alone (no f32 output, residual or "
                                 "peers), at most 8 copies, rows of ldc16 >= the width, a multiple of 8");
            for (int r = 0; r < g.n_c16; r++)
                if (!g.c16[r] || ((uintptr_t) g.c16[r] & 15) ||
                    !make_tmap_out16(&maps.c16[s][r], g.c16[r], M, g.n_out, g.ldc16))
                    return set_error("gemm: cannot build the TMA descriptor of a bf16 copy");
            p.n_c16 = g.n_c16;
        }
        pp.tile0[s] = tiles_n;
        tiles_n += (int) ((g.N + BN_T - 1) / BN_T);
    }
    pp.tile0[nseg] = tiles_n;
    pp.num_n = tiles_n;
    pp.raster = gp.raster;
    {
        // a function attribute holds per device: set it once on each
        static std::mutex mu;
        static uint64_t set_on = 0;
        int dev = 0;
        cudaGetDevice(&dev);
        std::lock_guard<std::mutex> lk(mu);
        if (dev >= 64 || !((set_on >> dev) & 1)) {
            if (cudaFuncSetAttribute(gemm_bf16_tc_pair_kernel<BN_T, false, NBUF>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, C::P_SMEM_BYTES) != cudaSuccess ||
                cudaFuncSetAttribute(gemm_bf16_tc_pair_kernel<BN_T, true, NBUF>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, C::P_SMEM_BYTES) != cudaSuccess)
                return check_launch("gemm (shared memory size)");
            if (dev < 64) set_on |= 1ull << dev;
        }
    }
    pp.dp_tiles = (int) gp.tiles;
    pp.sk_tiles = 0;
    pp.sk_q = 0;
    pp.sk_epoch = 0;
    const bool sk = gp.stream_k && sk_claim(st, &pp.sk_epoch);
    if (sk) {
        pp.dp_tiles = gp.dp_tiles;
        pp.sk_tiles = gp.sk_tiles;
        pp.sk_q = gp.sk_q;
    }
    // A stream-K launch's runs start at staggered k offsets, so a panel of
    // the streamed operand is read by its tiles at different times: it stays
    // in L2 without the evict-first hint (ZEST_GEMM_HINT=0/1 forces it).
    pp.stream_hint = !sk;
    if (const char *h = getenv("ZEST_GEMM_HINT")) pp.stream_hint = h[0] == '1';
    // stream-K spreads even a small launch over every pair
    const int max_pairs = num_sms() / 2;
    const int pairs = sk ? max_pairs : (int) (gp.tiles < max_pairs ? gp.tiles : max_pairs);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned) (2 * pairs));
    cfg.blockDim = dim3(NUM_THREADS);
    cfg.dynamicSmemBytes = C::P_SMEM_BYTES;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (sk)
        cudaLaunchKernelEx(&cfg, gemm_bf16_tc_pair_kernel<BN_T, true, NBUF>, ta, maps, pp);
    else
        cudaLaunchKernelEx(&cfg, gemm_bf16_tc_pair_kernel<BN_T, false, NBUF>, ta, maps, pp);
    if (sk) sk_release(st);
    return check_launch("gemm");
}

// The one-CTA kernel (128 x 256 tiles), for calls of at most 128 rows.
int launch_single(const CUtensorMap &ta, int64_t M, int64_t K, const gemm_seg &g, unsigned *err_flag,
                  cudaStream_t st) {
    CUtensorMap tb;
    if (!make_tmap(&tb, g.b, g.N, K, g.ldb, BN)) return set_error("gemm: cannot build the TMA descriptors");
    gemm_params p;
    memset(&p, 0, sizeof p);
    p.M = M;
    p.N = g.N;
    p.K = K;
    p.ldc = g.ldc;
    p.n_out = g.n_out;
    p.c = g.c;
    p.err = err_flag;
    p.mode = g.mode;
    p.resid = g.resid;
    p.ldr = g.ldr;
    p.a_next = g.a_next;
    p.lda_next = g.lda_next;
    p.c_mc = g.c_mc;
    p.mc_store = g.mc_store;
    p.num_m = (int) ((M + BM - 1) / BM);
    p.num_n = (int) ((g.N + BN - 1) / BN);
    p.num_k = (int) ((K + BK - 1) / BK);
    p.tma_store = 0;
    {
        static std::mutex mu;
        static uint64_t set_on = 0;  // per device, as the attribute holds
        int dev = 0;
        cudaGetDevice(&dev);
        std::lock_guard<std::mutex> lk(mu);
        if (dev >= 64 || !((set_on >> dev) & 1)) {
            if (cudaFuncSetAttribute(gemm_bf16_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) !=
                cudaSuccess)
                return check_launch("gemm (shared memory size)");
            if (dev < 64) set_on |= 1ull << dev;
        }
    }
    const int64_t tiles = (int64_t) p.num_m * p.num_n;
    const int grid = (int) (tiles < num_sms() ? tiles : num_sms());
    gemm_bf16_tc_kernel<<<grid, NUM_THREADS, SMEM_BYTES, st>>>(ta, tb, p);
    return check_launch("gemm");
}

}  // namespace

int launch_gemm_group(const uint16_t *a_bf16, int64_t lda, int64_t M, int64_t K, int nseg, gemm_seg *segs,
                      unsigned *err_flag, cudaStream_t st) {
    if (M <= 0 || nseg <= 0) return 0;
    if (nseg > MAX_SEG) return set_error("gemm: at most 4 weights in a group");
    if (!err_flag) return set_error("gemm: no device error word");
    if (K <= 0 || K % 8 || lda < K || lda % 8 || ((uintptr_t) a_bf16 & 15))
        return set_error("gemm: K and the row strides must be multiples of 8 and the operands 16-byte aligned");
    for (int s = 0; s < nseg; s++) {
        gemm_seg &g = segs[s];
        if (g.N <= 0 || g.ldb < K || g.ldb % 8 || ((uintptr_t) g.b & 15))
            return set_error("gemm: K and the row strides must be multiples of 8 and the operands 16-byte aligned");
        if (g.mode < MODE_F32 || g.mode > MODE_SWIGLU || (g.mode == MODE_SWIGLU && g.N % 16))
            return set_error("gemm: bad output mode");
        const int64_t width = g.mode == MODE_SWIGLU ? g.N / 2 : g.N;
        if (g.n_out <= 0 || g.n_out > width) g.n_out = width;
        if (!g.c && !g.a_next && !g.c_mc && !g.n_c16) return set_error("gemm: no output");
        if (g.c_mc && (g.c || g.mode == MODE_SWIGLU || g.resid || g.a_next || g.ldc < g.n_out))
            return set_error("gemm: a multicast output takes fp32 or bf16 results alone, rows of ldc >= the width");
        if (g.c && g.ldc < g.n_out) return set_error("gemm: ldc smaller than the output width");
        if (g.resid && (g.mode == MODE_SWIGLU || !g.c || g.ldr < g.n_out))
            return set_error("gemm: a residual needs an fp32 or bf16 output of its width");
        if (g.a_next && (g.mode != MODE_SWIGLU || g.n_out % 8 || g.lda_next < g.n_out || g.lda_next % 8 ||
                         ((uintptr_t) g.a_next & 15)))
            return set_error("gemm: the next operand needs SwiGLU, a width of 8s and 16-byte aligned rows");
        if (g.n_peers < 0 || g.n_peers > MAX_PEERS || (g.n_peers && !g.c_peers))
            return set_error("gemm: 0 to 7 peer copies, given by pointer");
        if (g.n_peers && (g.mode == MODE_SWIGLU || !g.c || g.ldc % 4 || ((uintptr_t) g.c & 15)))
            return set_error("gemm: peer copies need a TMA-stored output (fp32 or bf16, 16-byte aligned rows) "
                             "and at most 7 peers");
        for (int r = 0; r < g.n_peers; r++)
            if (!g.c_peers[r] || ((uintptr_t) g.c_peers[r] & 15))
                return set_error("gemm: a peer's copy must be 16-byte aligned");
        if (g.n_c16 < 0 || g.n_c16 > MAX_PEERS + 1 ||
            (g.n_c16 && (g.mode != MODE_BF16 || g.c || g.c_mc || g.resid || g.n_peers || !g.c16 ||
                         g.ldc16 < g.n_out || g.ldc16 % 8)))
            return set_error("gemm: bf16 copies take a bf16-mode output alone (no f32 output, residual or "
                             "peers), at most 8 copies, rows of ldc16 >= the width, a multiple of 8");
        for (int r = 0; r < g.n_c16; r++)
            if (!g.c16[r] || ((uintptr_t) g.c16[r] & 15))
                return set_error("gemm: a bf16 copy must be 16-byte aligned");
    }
    int64_t Ns[MAX_SEG];
    for (int s = 0; s < nseg; s++) Ns[s] = segs[s].N;
    gemm_plan gp;
    plan_gemm(M, K, nseg, Ns, 0, gp);
    CUtensorMap ta;
    if (!make_tmap(&ta, a_bf16, M, K, lda, BM)) return set_error("gemm: cannot build the TMA descriptors");
    if (!gp.pair) {
        for (int s = 0; s < nseg; s++)
            if (segs[s].n_peers > 0 || segs[s].n_c16 > 0)
                return set_error("gemm: peer and bf16 copies need more than 128 rows (the pair kernel)");
        for (int s = 0; s < nseg; s++)
            if (launch_single(ta, M, K, segs[s], err_flag, st)) return -1;
        return 0;
    }
    switch (gp.bn) {
        case 192: return launch_pair_group<192, 2>(ta, M, K, nseg, segs, gp, err_flag, st);
        case 160: return launch_pair_group<160, 2>(ta, M, K, nseg, segs, gp, err_flag, st);
        case 128: return launch_pair_group<128, 2>(ta, M, K, nseg, segs, gp, err_flag, st);
        default: return launch_pair_group<256, 2>(ta, M, K, nseg, segs, gp, err_flag, st);
    }
}

void plan_gemm(int64_t M, int64_t K, int nseg, const int64_t *Ns, int sms, gemm_plan &gp) {
    gp = gemm_plan{};
    if (sms <= 0) sms = num_sms();
    gp.num_k = (int) ((K + BK - 1) / BK);
    // The CTA-pair kernel unless ZEST_GEMM_PAIR=0 or the rows fit one 128-row tile.
    const char *pair_env = getenv("ZEST_GEMM_PAIR");
    gp.pair = M > BM && !(pair_env && pair_env[0] == '0');
    if (!gp.pair) {
        // one launch per weight, each its own tiles in groups of 8 tile rows
        gp.bn = BN;
        gp.num_m = (int) ((M + BM - 1) / BM);
        int64_t widest = 0;
        for (int s = 0; s < nseg; s++) {
            const int64_t n = (Ns[s] + BN - 1) / BN;
            gp.num_n += (int) n;
            widest = n > widest ? n : widest;
        }
        gp.tiles = (int64_t) gp.num_m * gp.num_n;
        const int64_t most = (int64_t) gp.num_m * widest;
        gp.ctas = (int) (most < sms ? most : sms);
        gp.raster = RASTER_GROUPS;
        gp.dp_tiles = (int) gp.tiles;
        return;
    }
    // 256-wide N tiles: measured on every shape of the configs, narrower
    // tiles lose 15-45 % per flop, more than they win back by rounding to
    // fewer waves. Narrower ones stay selectable for tests and tuning.
    gp.bn = 256;
    if (const char *force = getenv("ZEST_GEMM_BN")) {
        const int f = atoi(force);
        if (f == 192 || f == 160 || f == 128) gp.bn = f;
    }
    gp.num_m = (int) ((M + P_BM - 1) / P_BM);
    for (int s = 0; s < nseg; s++) gp.num_n += (int) ((Ns[s] + gp.bn - 1) / gp.bn);
    gp.tiles = (int64_t) gp.num_m * gp.num_n;
    // keep the re-read operand within about half of the 126 MB L2 (the rest
    // holds the streamed operand's tiles and the outputs on their way out)
    const double l2_budget = 60e6, a_bytes = 2.0 * (double) M * (double) K;
    double b_bytes = 0;
    for (int s = 0; s < nseg; s++) b_bytes += 2.0 * (double) Ns[s] * (double) K;
    gp.raster = b_bytes <= l2_budget && b_bytes <= a_bytes ? RASTER_ROWS
                : a_bytes <= l2_budget                     ? RASTER_COLS
                                                           : RASTER_GROUPS;
    if (const char *force = getenv("ZEST_GEMM_RASTER")) {
        const int f = atoi(force);
        if (f >= RASTER_GROUPS && f <= RASTER_COLS) gp.raster = f;
    }
    const int max_pairs = sms / 2;
    gp.dp_tiles = (int) gp.tiles;
    gp.stream_k = plan_stream_k(gp, max_pairs) ? 1 : 0;
    if (!gp.stream_k) {
        gp.dp_tiles = (int) gp.tiles;
        gp.sk_tiles = 0;
        gp.sk_q = 0;
    }
    // stream-K spreads even a small launch over every pair
    const int64_t pairs = gp.stream_k ? max_pairs : (gp.tiles < max_pairs ? gp.tiles : max_pairs);
    gp.ctas = (int) (2 * pairs);
}

int launch_gemm(const uint16_t *a_bf16, int64_t lda, const uint16_t *b_bf16, int64_t ldb, int64_t M, int64_t N,
                int64_t K, int mode, float *c, int64_t ldc, int64_t n_out, unsigned *err_flag, cudaStream_t st) {
    if (M <= 0 || N <= 0) return 0;
    gemm_seg g = { b_bf16, ldb, N, ldc, n_out, mode, c };
    return launch_gemm_group(a_bf16, lda, M, K, 1, &g, err_flag, st);
}

}  // namespace zest
