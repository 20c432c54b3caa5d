/*
 * Internal interface of the append-KV step (pgqa_append.cu), used by the C entry
 * points in pgqa_decode.cu.
 */
#ifndef PGQA_APPEND_H_
#define PGQA_APPEND_H_

#include <cuda_runtime.h>
#include <stdint.h>

namespace pgqa {

/* Bits of the device error word the append kernel may set (same word and meaning as
 * the decode kernel's). */
constexpr int32_t kAppendBadPage = 2;
constexpr int32_t kAppendBadSeqlen = 4;

struct AppendArgs {
    const uint4* k_new;      // [B, S_new, Hkv, 128] bf16 or e4m3, as 16-byte pieces
    const uint4* v_new;
    uint4* k_cache;          // [num_pages, P, Hkv, 128], same element type
    uint4* v_cache;
    const int32_t* seq_lens;     // lengths before the append
    const int32_t* block_table;  // [B, bt_stride]
    int32_t* err;                // device error word (may be null)
    int32_t B, S_new, Hkv, P, bt_stride, num_pages;
    int64_t cap_tokens;          // bt_stride * P
    int32_t row_pieces_log2;     // 16-byte pieces per token row: 4 (bf16, 256 B) or 3 (e4m3)
};

/* Launch on `stream` (programmatic dependent).  Returns 0, or -1 if the launch failed. */
int launch_append(const AppendArgs& a, int num_sms, cudaStream_t stream);

}  // namespace pgqa

#endif  // PGQA_APPEND_H_
