/*
 * Work partition of the paged-GQA decode, shared by the device kernel and the host
 * simulation (pgqa_simulate_partition), so the CPU tests check the exact
 * arithmetic the GPU runs.
 *
 * The reference splits each (batch, kv_head) unit into `ns` equal page ranges, with
 * ns picked from seven hand-tuned regimes on the *capacity* seqlen_k
 * (submission_clean.cu:375-430, :453-461), and lets splits beyond a sequence's real
 * length exit early (:93).  Here the work is instead measured in 16-token chunks
 * of the *actual* lengths and cut into equal contiguous slices:
 *
 *   unit u = (b, j), j in [0, units_per_seq) = (kv_head, group of row groups), b-major;
 *   unit (b, j) owns n_b = ceil(L_b / 16) chunks;
 *   flat chunk index of chunk c of unit (b, j) = pre[b] * U + j * n_b + c,
 *   where pre[b] = sum_{b' < b} n_b' and U = units_per_seq;
 *   T = pre[B] * U chunks in total.
 *
 * Active CTA i of n owns flat chunks [i*T/n, (i+1)*T/n); inside it, warp k of w owns
 * the k-th of w equal sub-slices.  Every chunk is owned by exactly one warp, every
 * warp gets the same number of chunks (+-1), and the number of pieces a unit is
 * cut into follows from its length, B*Hkv and the SM count.
 */
#ifndef PGQA_PARTITION_H_
#define PGQA_PARTITION_H_

#include <stdint.h>

#if defined(__CUDACC__)
#define PGQA_HD __host__ __device__ __forceinline__
#else
#define PGQA_HD inline
#endif

namespace pgqa {

constexpr int kChunkTokens = 16;   // tokens per pipeline stage / MMA M tile
constexpr int kHeadDim = 128;      // the only head dimension compiled
constexpr int kHeadsPerGroup = 8;  // query rows per MMA N tile (a row group)

PGQA_HD int64_t ceil_div64(int64_t a, int64_t b) { return (a + b - 1) / b; }

/* Chunks of a sequence of `len` valid tokens (clamped to [0, cap]). */
PGQA_HD int64_t seq_chunks(int64_t len, int64_t cap_tokens) {
    if (len < 0) len = 0;
    if (len > cap_tokens) len = cap_tokens;
    return ceil_div64(len, kChunkTokens);
}

/* Products below this bound fit 32-bit unsigned arithmetic (much cheaper on the GPU
 * than 64-bit division); the results are identical either way. */
constexpr int64_t kSmallProduct = 0xffffffffll;

/* Start of slice i when [0, total) is cut into n equal contiguous slices. */
PGQA_HD int64_t slice_begin(int64_t i, int64_t n, int64_t total) {
    if (i * total <= kSmallProduct) return (int64_t)((uint32_t)(i * total) / (uint32_t)n);
    return (i * total) / n;
}

/* Index of the slice that contains position x (0 <= x < total). */
PGQA_HD int64_t slice_owner(int64_t x, int64_t n, int64_t total) {
    const int64_t num = (x + 1) * n - 1;
    if (num <= kSmallProduct && total <= kSmallProduct)
        return (int64_t)((uint32_t)num / (uint32_t)total);
    return num / total;
}

/* Number of active CTAs for `total` chunks: every active warp gets at least
 * `min_chunks` chunks unless the whole problem is smaller than one CTA's share. */
PGQA_HD int64_t active_ctas(int64_t total, int64_t grid, int64_t warps, int64_t min_chunks) {
    const int64_t per = warps * min_chunks;
    int64_t n = (total <= kSmallProduct && per <= kSmallProduct)
                    ? (int64_t)((uint32_t)total / (uint32_t)per)
                    : total / per;
    if (n > grid) n = grid;
    if (n < 1) n = 1;
    return n;
}

/* Active CTAs when every unit has the same number of chunks (`uniform`): rounded down to
 * a multiple of the unit count, so that each unit is split over exactly k CTAs and no CTA
 * holds the end of one unit and the start of the next (one record and one arrival per
 * CTA instead of two).  Only when that idles at most 1/32 of the CTAs: c2 (16 units on
 * 148 SMs) runs on 144, nine CTAs per unit. */
PGQA_HD int64_t align_ctas(int64_t n, int64_t units, bool uniform) {
    if (!uniform || units <= 0 || n < units) return n;
    const int64_t aligned = (n / units) * units;
    return (n - aligned) * 32 <= n ? aligned : n;
}

/* Active warps of a CTA whose slice holds `len` chunks. */
PGQA_HD int64_t active_warps(int64_t len, int64_t warps) {
    return len < warps ? len : warps;
}

/* Global record slot of CTA c for unit starting at flat chunk `unit_begin`:
 * 2c when the unit contains the CTA's first chunk, else 2c+1. */
PGQA_HD int64_t record_slot(int64_t c, int64_t cta_begin, int64_t unit_begin) {
    return unit_begin <= cta_begin ? 2 * c : 2 * c + 1;
}

}  // namespace pgqa

#endif  // PGQA_PARTITION_H_
