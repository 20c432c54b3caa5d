/*
 * pgqa_append.cu - append-KV step: write each sequence's new key/value tokens into its
 * pages before the decode reads them.
 *
 * flash_attn_with_kvcache(q, k_cache, v_cache, k, v, cache_seqlens, block_table, ...)
 * -- the operator the reference is judged against (task.md:16-26, where it is called
 * with k = v = None) -- writes k/v [B, S_new, Hkv, D] at token positions
 * [L_b, L_b + S_new) of sequence b (L_b = cache_seqlens[b], the length before the
 * append) and then attends over L_b + S_new keys.  Token t of sequence b lives in slot
 * t % P of page block_table[b, t / P] (task.md:94,146), one row per KV head.
 *
 * The step is a scatter of token rows (256 bytes for bf16 pools, 128 for e4m3): each
 * thread moves one 16-byte piece of K and the same piece of V, so a warp writes whole
 * rows (coalesced runs) and reads k/v in their contiguous order.  It launches as a
 * programmatic dependent and waits (griddepcontrol.wait) before touching memory, so it
 * may overlap the previous
 * kernel's tail without racing its reads of the pool.  Rows whose position lies past
 * the table's capacity, or whose page id is outside [0, num_pages), are skipped and
 * flagged in the device error word.
 */
#include <cuda_runtime.h>
#include <stdint.h>

#include "pgqa_append.h"
#include "pgqa_ptx.cuh"

namespace pgqa {

namespace {

constexpr int kAppendThreads = 256;

__global__ void __launch_bounds__(kAppendThreads)
append_kv_kernel(const AppendArgs a) {
    ptx::griddep_wait();
    const int sh = a.row_pieces_log2;
    const int64_t total = ((int64_t)a.B * a.S_new * a.Hkv) << sh;
    const int64_t stride = (int64_t)gridDim.x * kAppendThreads;
    int32_t bad = 0;
    for (int64_t x = (int64_t)blockIdx.x * kAppendThreads + threadIdx.x; x < total; x += stride) {
        const int64_t row = x >> sh;              // (b, s, kvh) row of k_new / v_new
        const int piece = (int)(x & ((1 << sh) - 1));
        const int32_t kvh = (int32_t)(row % a.Hkv);
        const int64_t bs = row / a.Hkv;
        const int32_t s = (int32_t)(bs % a.S_new);
        const int32_t b = (int32_t)(bs / a.S_new);
        const int32_t L0 = __ldg(a.seq_lens + b);
        const int64_t t = (int64_t)L0 + s;
        if (L0 < 0 || t >= a.cap_tokens) { bad |= kAppendBadSeqlen; continue; }
        const int32_t pid = __ldg(a.block_table + (int64_t)b * a.bt_stride + t / a.P);
        if (pid < 0 || pid >= a.num_pages) { bad |= kAppendBadPage; continue; }
        const int64_t dst = ((((int64_t)pid * a.P + t % a.P) * a.Hkv + kvh) << sh) + piece;
        const uint4 kv = __ldg(a.k_new + x);
        const uint4 vv = __ldg(a.v_new + x);
        a.k_cache[dst] = kv;
        a.v_cache[dst] = vv;
    }
    if (bad && a.err != nullptr) atomicOr(a.err, bad);
}

}  // namespace

int launch_append(const AppendArgs& a, int num_sms, cudaStream_t stream) {
    const int64_t total = ((int64_t)a.B * a.S_new * a.Hkv) << a.row_pieces_log2;
    if (total == 0) return 0;
    int64_t blocks = (total + kAppendThreads - 1) / kAppendThreads;
    const int64_t cap = (int64_t)num_sms * 8;  // 8 resident 256-thread CTAs per SM
    if (blocks > cap) blocks = cap;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)blocks);
    cfg.blockDim = dim3(kAppendThreads);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, append_kv_kernel, a) != cudaSuccess) {
        cudaGetLastError();
        return -1;
    }
    return 0;
}

}  // namespace pgqa
