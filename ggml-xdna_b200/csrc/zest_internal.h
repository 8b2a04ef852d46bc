// Internal declarations shared by the CUDA sources of libzest_b200.so.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace zest {

// ggml_type ids (GGUF file-format values) of the weight types converted
enum {
    TYPE_F32 = 0,
    TYPE_F16 = 1,
    TYPE_Q8_0 = 8,
    TYPE_Q4_K = 12,
    TYPE_Q6_K = 14,
    TYPE_IQ3_S = 21,
};

// GEMM output modes (kernels/bfp16_gemm/aie_kernels/aie2p/mm_bfp_acc.cc:138-148)
enum {
    MODE_F32 = 0,     // fp32 as accumulated
    MODE_BF16 = 1,    // every value rounded to bf16, nearest even
    MODE_SWIGLU = 2,  // SiLU(gate) * up, rounded to bf16 (weights interleaved 8 gate + 8 up rows)
};

// Records `msg` as the thread's last error and returns -1.
int set_error(const char *msg);
// After a launch: -1 with the CUDA error recorded, or 0.
int check_launch(const char *what);
bool iq3s_grid_loaded();
int set_iq3s_grid(const uint32_t *grid512);

int launch_pack_activations(const float *x, int64_t T, int64_t K, int64_t ldx, int64_t m_pad, uint8_t *a_bytes,
                            uint16_t *a_bf16, int64_t ldb, cudaStream_t st);

int launch_convert_weight(int type, const void *src0, const void *src1, int fused, int64_t n_rows, int64_t src_row0,
                          int64_t src_rows_total, int64_t K, int64_t n_pad, uint8_t *b_bytes, uint16_t *b_bf16,
                          cudaStream_t st);

// One weight of a grouped GEMM: its B operand (N rows), output and mode,
// and what the epilogue fuses: a residual added to the result (the ADD
// after o and down), or for SwiGLU the next GEMM's A operand (the bf16 copy
// of the result's bfp16 rounding, as K2 would pack it).
struct gemm_seg {
    const uint16_t *b;
    int64_t ldb, N, ldc, n_out;  // n_out <= 0: all (N, or N/2 for SwiGLU)
    int mode;
    float *c;                    // may be null for SwiGLU with a_next
    const float *resid = nullptr;
    int64_t ldr = 0;
    uint16_t *a_next = nullptr;
    int64_t lda_next = 0;
    float *c_mc = nullptr;       // multicast address: results added into every GPU's copy (NVSwitch reduction)
    int mc_store = 0;            // with c_mc: stored into every copy instead (an N-shard's all-gather)
    float *const *c_peers = nullptr;  // the tiles also stored into these (other GPUs' buffers laid out as c)
    int n_peers = 0;
    uint16_t *const *c16 = nullptr;   // bf16 copies of the tiles (bf16 mode): [M][ldc16] each
    int n_c16 = 0;
    int64_t ldc16 = 0;
};

// How K3 runs one launch: the kernel, its tiles, the order the persistent
// CTAs walk them in, and the stream-K split of the last waves.
struct gemm_plan {
    int pair;                // 1: CTA pairs on 256-row tiles; 0: one CTA per 128-row tile
    int bn;                  // output tile width
    int num_m, num_n, num_k; // tile rows, tile columns (all weights end to end), 64-wide k-blocks
    int64_t tiles;
    int ctas;                // CTAs launched (the one-CTA kernel: per weight, at most)
    int raster;              // 0: groups of 8 tile rows, 1: rows (A streamed), 2: columns (B streamed)
    int stream_k;            // 1: the last waves are cut into runs of k-blocks
    int dp_tiles, sk_tiles;  // tiles run whole; tiles cut into runs
    int64_t sk_q;            // k-blocks per pair over the cut tiles
};

// The plan of a launch of A [M][K] against nseg weights of Ns rows each on
// `sms` SMs (<= 0: this device's, capped by ZEST_GEMM_MAX_SMS). Reads the
// tuning variables (ZEST_GEMM_PAIR, _BN, _RASTER, _SK) as the launch does.
void plan_gemm(int64_t M, int64_t K, int nseg, const int64_t *Ns, int sms, gemm_plan &gp);

// Up to 4 weights sharing one A (q, k and v; gate and up) in one launch.
int launch_gemm_group(const uint16_t *a_bf16, int64_t lda, int64_t M, int64_t K, int nseg, gemm_seg *segs,
                      unsigned *err_flag, cudaStream_t st);

// n_out: output columns to write (<= 0: all, N or N/2 for SwiGLU); a fused
// gate/up copy padded to f_pad writes only the real F.
int launch_gemm(const uint16_t *a_bf16, int64_t lda, const uint16_t *b_bf16, int64_t ldb, int64_t M, int64_t N,
                int64_t K, int mode, float *c, int64_t ldc, int64_t n_out, unsigned *err_flag, cudaStream_t st);

}  // namespace zest
