/*
 * pgqa_tc.h - the tensor-core (tcgen05 / TMEM) variant of the paged-GQA decode, used for
 * the paths whose mma.sync form is bound by instruction issue: e4m3 KV pages and several
 * query tokens per sequence.  Host-side interface for pgqa_decode.cu.
 */
#ifndef PGQA_TC_H_
#define PGQA_TC_H_

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace pgqa {

struct TcParams {
    const __nv_bfloat16* q;     // [B, Sq, Hq, 128]
    __nv_bfloat16* out;         // [B, Sq, Hq, 128]
    float* lse_out;             // optional [B, Hq, Sq] natural-log sum-exp per query row
    const int32_t* seq_lens;
    const int32_t* block_table;
    void* rec_o;                // [2 * grid] records of normalised O (fp32 at 16 rows, bf16 at 32)
    float* rec_lse;             // [2 * grid][rows] log2-sum-exp
    int32_t* counters;          // [B * Hkv] arrival counters (zero between calls)
    int32_t* err;               // device error word
    int32_t B, Hq, Hkv, g, Sq;
    int32_t rows;               // query rows per KV head = g * Sq (row r: head r / Sq, token r % Sq)
    int32_t causal;             // query token i sees keys [0, L - Sq + i] instead of [0, L)
    int32_t len_add;            // tokens appended by this call
    const float* k_scale;       // e4m3 pools: dequantisation factor per KV head (null = 1)
    const float* v_scale;
    int32_t page_size, bt_stride, num_pages;
    int32_t page_shift;         // log2(page_size) when it is a power of two, else -1
    int64_t cap_tokens;         // bt_stride * page_size
    float scale_log2;           // scale * log2(e)
    int32_t min_chunks;         // lower bound on 16-token chunks per active CTA
    int32_t debug_stuck;        // test hook: > 0 makes CTA 0's first stage expect 16 bytes too many
    uint64_t wait_limit_ns;     // bound on every wait
};

/* Query rows per KV head the tensor-core variant handles (N of its MMAs, padded to 16). */
constexpr int kTcMaxRows = 32;

/* Dynamic shared memory of the variant for B sequences (e4m3 or bf16 pools, rows <= 32). */
size_t tc_smem_bytes(bool kv8, int rows, int64_t B);

/* Launches the variant (persistent grid of `grid` CTAs); returns 0 or a CUDA error. */
cudaError_t launch_tc(const CUtensorMap& kmap, const CUtensorMap& vmap, const TcParams& p,
                      bool kv8, int grid, size_t smem, bool pdl, cudaStream_t stream);

}  // namespace pgqa

#endif  // PGQA_TC_H_
