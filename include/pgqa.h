/*
 * pgqa.h - C ABI of the B200 (sm_100a) paged grouped-query-attention decode library
 * (libpgqa.so).
 *
 * The library computes, for every sequence b and query head h,
 *
 *     kv       = h / (num_heads / num_heads_k)
 *     tokens   = the first seq_lens[b] tokens of the paged cache of sequence b,
 *                token t living in page block_table[b, t / page_size] at slot t % page_size
 *     out[b,h] = softmax(scale * q[b,h] . K[tokens, kv]^T) . V[tokens, kv]
 *
 * with bf16 inputs/outputs and fp32 accumulation.  Layouts (all contiguous):
 *     q, out        [B, Sq, Hq, D]  (Sq = 1 for decode) bf16
 *     k, v pools    [num_pages, page_size, Hkv, D]   bf16
 *     seq_lens      [B]                              int32
 *     block_table   [B, bt_stride]                   int32
 *
 * Only the first ceil(seq_lens[b] / page_size) entries of a block-table row are
 * ever read; padding slots may hold any value.
 *
 * All entry points are asynchronous with respect to the host (no device
 * synchronisation inside), except the ones documented as "synchronous".
 */
#ifndef PGQA_H_
#define PGQA_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes returned by the int-returning entry points. */
enum pgqa_status {
    PGQA_OK = 0,
    PGQA_ERR_NULL_POINTER = 1,      /* a required pointer is NULL                       */
    PGQA_ERR_BAD_SHAPE = 2,         /* B/Hq/Hkv/D/page_size/num_pages/stride invalid    */
    PGQA_ERR_UNSUPPORTED = 3,       /* valid but not implemented (D != 128, P % 16 ...) */
    PGQA_ERR_MISALIGNED = 4,        /* a pointer violates the alignment contract        */
    PGQA_ERR_WORKSPACE = 5,         /* workspace missing / too small / allocation failed */
    PGQA_ERR_CUDA = 6,              /* a CUDA runtime/driver call failed                */
    PGQA_ERR_NO_DEVICE = 7,         /* no usable CUDA device (or not sm_100)            */
    PGQA_ERR_DEVICE_TIMEOUT = 8,    /* a bounded device-side wait expired (device word) */
    PGQA_ERR_DEVICE_BAD_PAGE = 9,   /* a block-table entry was outside [0, num_pages)   */
    PGQA_ERR_DEVICE_BAD_SEQLEN = 10, /* a seq_len was < 0 or above the table capacity   */
    PGQA_ERR_SCRATCH_LIMIT = 11     /* shape exceeds pgqa_decode_noalloc's fixed scratch */
};

/*
 * Reference drop-in.  Replaces `extern "C" void run_kernel(...)` of the MetaX C500
 * submission (submission_clean.cu:432-447; contract task.md:33-54), with the same
 * symbol name, argument types, order and meaning:
 *   block_table row width = num_blocks / batch_size, pool size = num_blocks pages,
 *   scale = 1/sqrt(headdim), launches on the legacy default stream, returns void.
 * Errors (which the reference ignores) are recorded and can be read back with
 * pgqa_last_status().  The first call on a device allocates the library's
 * per-device workspace (cudaMalloc), so the first call must not be inside a
 * CUDA-graph capture.  Like the reference's static buffers, that workspace is shared
 * by every run_kernel call on the device: calls that may overlap on the GPU (several
 * streams or host threads) must use pgqa_decode_v1/_v2 with a workspace each.
 * Beyond the reference (which fixes seqlen_q = 1, causal = 0; task.md:64-66),
 * seqlen_q >= 1 query tokens per sequence are accepted, q and output being
 * (B, seqlen_q, Hq, D); with causal = 1 token i sees keys [0, L - seqlen_q + i].
 */
void run_kernel(const void* q, const void* k_cache_paged, const void* v_cache_paged,
                void* output, const int32_t* cache_seqlens, const int32_t* block_table,
                int64_t batch_size, int64_t seqlen_k, int64_t seqlen_q, int64_t num_heads,
                int64_t num_heads_k, int64_t headdim, int64_t page_block_size,
                int64_t num_blocks, int64_t causal);

/*
 * Extended entry point (no counterpart symbol in the reference; it generalises
 * run_kernel, submission_clean.cu:432-504, for pools whose page count is not
 * batch_size * table width and for an explicit scale/stream).
 *   num_pages   : pages in each K/V pool (TMA bounds; entries >= num_pages are errors)
 *   bt_stride   : block_table row stride in int32 elements
 *   max_seqlen  : capacity bound in tokens (<= bt_stride * page_size); 0 = derive
 *   scale       : softmax scale (e.g. 1/sqrt(D))
 *   workspace   : device buffer of >= pgqa_workspace_size(...) bytes, zero-filled
 *                 once before first use (pgqa_workspace_init); the kernel leaves it
 *                 zeroed.  NULL = use the library's per-device workspace.
 *   stream      : cudaStream_t (NULL = legacy default stream)
 * Calls that share one workspace must be ordered on one stream.
 */
int pgqa_decode_v1(const void* q, const void* k_cache, const void* v_cache, void* out,
                   const int32_t* seq_lens, const int32_t* block_table, int64_t batch_size,
                   int64_t num_heads, int64_t num_heads_k, int64_t headdim,
                   int64_t page_size, int64_t num_pages, int64_t bt_stride,
                   int64_t max_seqlen, float scale, void* workspace, size_t workspace_bytes,
                   void* stream);

/*
 * pgqa_decode_v1 with seqlen_q query tokens per sequence (no counterpart symbol in the
 * reference; the ABI run_kernel already carries seqlen_q and causal, task.md:40-53).
 * q and out are [B, seqlen_q, Hq, D]; query token i of sequence b sees keys
 * [0, L_b) or, with causal = 1, [0, L_b - seqlen_q + i] (a query with no visible key
 * gives zeros).  The workspace must hold pgqa_workspace_size_v2(...) bytes.
 */
int pgqa_decode_v2(const void* q, const void* k_cache, const void* v_cache, void* out,
                   const int32_t* seq_lens, const int32_t* block_table, int64_t batch_size,
                   int64_t seqlen_q, int64_t num_heads, int64_t num_heads_k, int64_t headdim,
                   int64_t page_size, int64_t num_pages, int64_t bt_stride, int64_t max_seqlen,
                   int64_t causal, float scale, void* workspace, size_t workspace_bytes,
                   void* stream);

/*
 * Append-KV step (no counterpart symbol in the reference; it is the k / v argument pair
 * of flash_attn_with_kvcache, which the reference's task passes as None, task.md:16-26).
 * Writes k_new / v_new [B, seqlen_new, Hkv, D] bf16 into the pools at token positions
 * [L_b, L_b + seqlen_new) of each sequence, L_b = seq_lens[b] being the length BEFORE
 * the append; token t goes to slot t % P of page block_table[b, t / P].  seq_lens is
 * not modified (the caller advances it).  Positions past the table capacity or page ids
 * outside [0, num_pages) are skipped and flagged in the device error word of
 * `workspace` (the library's own when NULL; read with pgqa_check_device_error).
 * Asynchronous on `stream`.
 */
int pgqa_append_kv(const void* k_new, const void* v_new, void* k_cache, void* v_cache,
                   const int32_t* seq_lens, const int32_t* block_table, int64_t batch_size,
                   int64_t seqlen_new, int64_t num_heads_k, int64_t headdim, int64_t page_size,
                   int64_t num_pages, int64_t bt_stride, void* workspace, void* stream);

/*
 * pgqa_append_kv followed by pgqa_decode_v2 over the extended sequences, in one call
 * (flash_attn_with_kvcache with k / v given; no counterpart symbol in the reference).
 * Sequence b is attended over L_b + seqlen_new keys; with causal = 1 query token i sees
 * keys [0, L_b + seqlen_new - seqlen_q + i].  seqlen_new = 0 is plain pgqa_decode_v2.
 */
int pgqa_decode_kvcache(const void* q, void* k_cache, void* v_cache, const void* k_new,
                        const void* v_new, void* out, const int32_t* seq_lens,
                        const int32_t* block_table, int64_t batch_size, int64_t seqlen_q,
                        int64_t seqlen_new, int64_t num_heads, int64_t num_heads_k,
                        int64_t headdim, int64_t page_size, int64_t num_pages, int64_t bt_stride,
                        int64_t max_seqlen, int64_t causal, float scale, void* workspace,
                        size_t workspace_bytes, void* stream);

/*
 * FP8 KV pages (no counterpart in the reference, whose pools are bf16).  k_cache and
 * v_cache hold float8 e4m3 (OCP "e4m3fn": bias 7, no infinities) in the same
 * [num_pages, P, Hkv, D] layout, one byte per element; the value of an element of KV
 * head h is e4m3 * k_scale[h] (resp. v_scale[h]) -- k_scale / v_scale are device arrays
 * of Hkv floats, NULL meaning 1.  q and out stay bf16 [B, seqlen_q, Hq, D].  k_new /
 * v_new (e4m3, [B, seqlen_new, Hkv, D], NULL when seqlen_new = 0) are appended first, as
 * in pgqa_decode_kvcache.  Everything else is pgqa_decode_v2 / pgqa_decode_kvcache; the
 * workspace size is pgqa_workspace_size_v2's.
 */
int pgqa_decode_fp8(const void* q, void* k_cache, void* v_cache, const void* k_new,
                    const void* v_new, void* out, const int32_t* seq_lens,
                    const int32_t* block_table, int64_t batch_size, int64_t seqlen_q,
                    int64_t seqlen_new, int64_t num_heads, int64_t num_heads_k, int64_t headdim,
                    int64_t page_size, int64_t num_pages, int64_t bt_stride, int64_t max_seqlen,
                    int64_t causal, float scale, const float* k_scale, const float* v_scale,
                    void* workspace, size_t workspace_bytes, void* stream);

/*
 * Every option in one call, with an optional log-sum-exp output (no counterpart in the
 * reference; flash_attn_with_kvcache's return_softmax_lse).  Fields not named below are
 * those of pgqa_decode_fp8 / pgqa_decode_kvcache, with the same meaning and checks.
 *   struct_size  sizeof(pgqa_decode_args) as the caller was compiled (checked)
 *   kv_format    0: bf16 pools (k_scale / v_scale must be NULL), 1: e4m3 pools
 *   softmax_lse  NULL, or fp32 [batch_size, num_heads, seqlen_q]: ln of the sum of
 *                exp(scale * q.k) over the keys each query row sees (-inf for a row that
 *                sees none).  Compiled for the default launch shape only: under the
 *                PGQA_WARPS / PGQA_STAGES sweep knobs a call asking for it returns
 *                PGQA_ERR_UNSUPPORTED.
 * The workspace size is pgqa_workspace_size_v2's; workspace NULL uses the library's.
 */
typedef struct pgqa_decode_args {
    size_t struct_size;
    const void* q;
    void* k_cache;
    void* v_cache;
    const void* k_new;
    const void* v_new;
    void* out;
    float* softmax_lse;
    const int32_t* seq_lens;
    const int32_t* block_table;
    int64_t batch_size, seqlen_q, seqlen_new, num_heads, num_heads_k, headdim;
    int64_t page_size, num_pages, bt_stride, max_seqlen, causal;
    float scale;
    int32_t kv_format;
    const float* k_scale;
    const float* v_scale;
    void* workspace;
    size_t workspace_bytes;
} pgqa_decode_args;

int pgqa_decode_ex(const pgqa_decode_args* args, void* stream);

/* pgqa_append_kv for e4m3 pools (128-byte token rows). */
int pgqa_append_kv_fp8(const void* k_new, const void* v_new, void* k_cache, void* v_cache,
                       const int32_t* seq_lens, const int32_t* block_table, int64_t batch_size,
                       int64_t seqlen_new, int64_t num_heads_k, int64_t headdim,
                       int64_t page_size, int64_t num_pages, int64_t bt_stride, void* workspace,
                       void* stream);

/*
 * Allocation-free variant of pgqa_decode_v1 (no counterpart in the reference).
 *
 * Some callers cannot allocate device memory when they call the decode: serving
 * engines that reserve nearly all of HBM in their own pool and allow no other
 * allocation on the hot path (cudaMalloc may also synchronise the device, which stalls
 * every stream), and plugin hosts that hand the operator only its input and output
 * buffers and have no workspace to give.  This entry point takes the same arguments as
 * pgqa_decode_v1 minus the workspace and allocates nothing: its scratch (split records
 * and arrival counters) lives in a fixed 4 MiB device array inside the library, which
 * every GPU that loads the library holds until the process exits.  The caller still
 * passes q, the pools, seq_lens, block_table and out.
 *
 * Limit: after the split records of a 148-SM B200 (2.58 MB) the array holds 50,552
 * arrival-counter entries, one per (sequence, unit, row group):
 *     batch_size * num_heads_k * G <= 50,552,
 *     G = 1 for up to 8 query heads per KV head, else 2 * ceil(ceil(g / 8) / 2)
 * (g = num_heads / num_heads_k): about 50,500 sequence x KV-head pairs at g <= 8,
 * 25,200 at g = 16, 12,600 at g = 32, 6,300 at g = 64.  The exact test is
 * pgqa_make_plan(...).workspace_bytes <= 4 MiB.  Larger shapes are rejected with
 * PGQA_ERR_SCRATCH_LIMIT before anything is launched.
 *
 * The first call on a device looks up the array's device address (once per device,
 * with that device current) and clears its error word; make that first call before
 * any stream capture.  Each call clears the arrival counters.  All calls share the one
 * array, so calls that overlap on the GPU (different streams, or different host
 * threads) race and give wrong results: order them on one stream.  Device-side errors
 * (bad page id, length above capacity, expired wait) are kept in the array's error
 * word until pgqa_noalloc_check_device_error reads them.
 */
int pgqa_decode_noalloc(const void* q, const void* k_cache, const void* v_cache, void* out,
                        const int32_t* seq_lens, const int32_t* block_table,
                        int64_t batch_size, int64_t num_heads, int64_t num_heads_k,
                        int64_t headdim, int64_t page_size, int64_t num_pages,
                        int64_t bt_stride, int64_t max_seqlen, float scale, void* stream);

/* Synchronous: waits for `stream`, then reads and clears the device-side error word that
 * pgqa_decode_noalloc calls on the current device share (no counterpart in the
 * reference).  Returns PGQA_OK (also when no such call has run on this device) or one
 * of the PGQA_ERR_DEVICE_* codes.  Allocates nothing. */
int pgqa_noalloc_check_device_error(void* stream);

/* Bytes of workspace pgqa_decode_v1 needs for this shape on the current device
 * (no counterpart in the reference, whose workspace is a hidden static buffer,
 * submission_clean.cu:478-491).  Returns 0 on invalid or unsupported shapes;
 * pgqa_last_status() then holds the reason. */
size_t pgqa_workspace_size(int64_t batch_size, int64_t num_heads, int64_t num_heads_k,
                           int64_t headdim, int64_t page_size);

/* Workspace bytes for pgqa_decode_v2 with seqlen_q query tokens (no counterpart in
 * the reference).  Returns 0 on invalid or unsupported shapes; pgqa_last_status() then
 * holds the reason. */
size_t pgqa_workspace_size_v2(int64_t batch_size, int64_t seqlen_q, int64_t num_heads,
                              int64_t num_heads_k, int64_t headdim, int64_t page_size);

/* Zero a caller-provided workspace on `stream` (asynchronous). */
int pgqa_workspace_init(void* workspace, size_t workspace_bytes, void* stream);

/* Status of the most recent run_kernel / pgqa_decode_v1 call on this host thread. */
int pgqa_last_status(void);

/* Human-readable text for a status code (static storage). */
const char* pgqa_status_string(int status);

/* Synchronous: waits for `stream`, reads and clears the device-side error word of
 * `workspace` (NULL = the library workspace of the current device).  Returns
 * PGQA_OK or one of the PGQA_ERR_DEVICE_* codes. */
int pgqa_check_device_error(void* workspace, void* stream);

/*
 * Launch plan (host-only, no GPU needed).  Reproduces the decisions the launcher
 * makes for a shape: replaces the reference's choose_num_splits
 * (submission_clean.cu:375-430) and its page rounding (:453-461).
 */
typedef struct pgqa_plan {
    int32_t grid_ctas;        /* persistent CTAs launched (one per SM)               */
    int32_t warps_per_cta;    /* streaming warps per CTA                              */
    int32_t stages;           /* TMA ring depth per warp (16-token stages)            */
    int32_t min_chunks_per_warp; /* lower bound on work per active warp (chunks)      */
    int32_t head_groups;      /* groups of <= 8 query rows per KV head               */
    int32_t units_per_seq;    /* num_heads_k * ceil(head_groups / groups_per_unit)    */
    int32_t smem_bytes;       /* dynamic shared memory per CTA                        */
    int32_t status;           /* PGQA_OK or why the shape cannot run                  */
    int64_t workspace_bytes;  /* pgqa_workspace_size for this shape                   */
    int32_t groups_per_unit;  /* row groups one warp carries over each K/V tile (1, 2) */
    int32_t reserved;
} pgqa_plan;

/* Fill *plan for a shape on a device with `num_sms` SMs and `smem_per_block_optin`
 * bytes of opt-in shared memory (pass 0, 0 to use B200 values: 148, 232448). */
int pgqa_make_plan(int64_t batch_size, int64_t num_heads, int64_t num_heads_k,
                   int64_t headdim, int64_t page_size, int32_t num_sms,
                   int32_t smem_per_block_optin, pgqa_plan* plan);

/*
 * Host simulation of the device work partition for given seq_lens (host array).
 * For each unit u = (b, kv, head_group) (b-major, B * units_per_seq entries) it
 * writes the number of CTAs whose slice intersects the unit (ctas_per_unit) and
 * the number of warp segments it is cut into (segments_per_unit), and returns the
 * number of active CTAs.  Used by the CPU tests to check that the split is exact
 * (every 16-token chunk is owned by exactly one warp).  Returns < 0 on error.
 */
int64_t pgqa_simulate_partition(const int32_t* seq_lens, int64_t batch_size,
                                int64_t units_per_seq, int64_t bt_capacity_tokens,
                                const pgqa_plan* plan, int32_t* ctas_per_unit,
                                int32_t* segments_per_unit);

/* Library build identifier (static storage). */
const char* pgqa_version(void);

#ifdef __cplusplus
}
#endif

#endif /* PGQA_H_ */
