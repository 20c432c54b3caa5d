/*
 * pgqa_decode.cu - paged grouped-query-attention decode for B200 (sm_100a).
 *
 * Replaces, behind the same `run_kernel` C symbol, the reference's
 *   - split-KV partial kernel   paged_gqa_mma_kernel   (submission_clean.cu:66-300;
 *     online-softmax form paged_gqa_decode_mma, optimized_c500_flash_attn.cu:463-664)
 *   - split combine             combine_kernel         (submission_clean.cu:307-360;
 *     LSE form combine_splits, optimized_c500_flash_attn.cu:666-728)
 *   - split-count policy        choose_num_splits      (submission_clean.cu:375-430)
 *   - host prologue / launcher  run_kernel             (submission_clean.cu:432-504)
 *
 * Design (one launch per call):
 *   * Persistent grid, one CTA per SM, W streaming warps per CTA.  The total work,
 *     measured in 16-token chunks of the *actual* sequence lengths, is cut into equal
 *     contiguous slices per CTA and per warp (pgqa_partition.h).  The per-unit split
 *     count therefore follows from B*Hkv, the lengths and the SM count; there are no
 *     per-case constants and no empty splits.
 *   * Each warp owns an S-stage ring of 8 KB stages in shared memory.  Lane 0 issues
 *     four TMA tile loads per stage (K and V, two 64-dim halves each, 16 tokens of one
 *     KV head, 128-byte swizzle) that complete on the stage's mbarrier.  Page ids come
 *     from a 32-entry block-table window loaded by the whole warp; only the first
 *     ceil(L_b / page_size) entries of a row are ever read.
 *   * Math per 16-token stage, tokens in the MMA M dimension ("swap AB"), 8 query rows
 *     of one KV head in N (a row group; with seqlen_q tokens a row is a (head, token)
 *     pair; with several row groups per KV head a warp carries two over each tile):
 *     S^T = K.Q^T (8 x mma.m16n8k16 bf16), fp32 online softmax in the log2 domain
 *     (scale*log2e folded into one multiply, ex2.approx, a reference max that moves
 *     only when a score exceeds it by 2^8), P^T moved into the B-operand layout with
 *     movmatrix.trans, O^T += V^T.P^T (8 x mma).
 *   * e4m3 pools (KV8): 4 KB stages, one 128-byte box each for K and V; the bytes are
 *     converted exactly to f16 after ldmatrix and multiplied with f16 MMAs, two chunks
 *     per step.
 *   * A unit (b, kv, row groups) that lies inside one warp's slice is normalised and
 *     stored as bf16 directly.  Units cut by warp boundaries are merged in shared
 *     memory at the end of the CTA; units cut by CTA boundaries write an fp32 record
 *     (o, log2-sum-exp) to the workspace, and the last CTA to finish the unit (atomic
 *     counter, reset by that CTA) merges the records -- the LSE combine, fused.
 *   * Launched as a programmatic dependent (griddepcontrol): the prologue overlaps the
 *     previous kernel's tail.  For calls long enough to repay it, each CTA cuts the
 *     work from a first read of the lengths and prefetches its warps' first chunks
 *     into L2 before griddepcontrol.wait (L2-only accesses; lengths, table and K/V
 *     are read again after the wait); nothing else touches global memory before the
 *     previous kernel completes.
 */
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <math.h>
#include <stddef.h>
#include <mutex>
#include <type_traits>

#include "../../include/pgqa.h"
#include "pgqa_append.h"
#include "pgqa_partition.h"
#include "pgqa_ptx.cuh"
#include "pgqa_tc.h"

namespace pgqa {

/* ------------------------------------------------------------------------------------ */
/* Device side                                                                          */
/* ------------------------------------------------------------------------------------ */

constexpr int kStageBytes = 8192;          // K (2 x 2 KB halves) + V (2 x 2 KB halves)
constexpr int kHalfBytes = 2048;           // 16 tokens x 64 dims x bf16
constexpr int kStageBytesKv8 = 4096;       // FP8 pools: K (16 tokens x 128 B) + V
constexpr float kLazyLog2 = 8.f;           // softmax reference max moves only beyond 2^8
constexpr uint64_t kWaitLimitNs = 1000000000ull;  // 1 s bound on any single wait

enum DeviceErr : int32_t { kErrTimeout = 1, kErrBadPage = 2, kErrBadSeqlen = 4 };
static_assert(kErrBadPage == kAppendBadPage && kErrBadSeqlen == kAppendBadSeqlen,
              "the append step shares the decode's error word");

struct DecodeParams {
    const __nv_bfloat16* q;
    __nv_bfloat16* out;
    float* lse_out;      // optional [B, Hq, Sq] fp32 natural-log sum-exp per query row
    const int32_t* seq_lens;
    const int32_t* block_table;
    float* rec_o;        // [2 * grid * NG][8 M tiles][32 lanes] float4 (O^T fragments)
    float* rec_lse;      // [2 * grid * NG][8 M tiles][8 heads]
    int32_t* counters;   // [B * U * NG][8 M tiles] arrival counters
    int32_t* err;        // device error word
    // n_hg groups of 8 query rows per KV head; a unit carries NG of them (n_w units per
    // KV head, U = Hkv * n_w per sequence): row group hg = w * NG + grp
    int32_t B, Hq, Hkv, g, n_hg, n_w, U;
    int32_t Sq;      // query tokens per sequence
    int32_t rows;    // query rows per KV head = g * Sq (row r: head r / Sq, token r % Sq)
    int32_t causal;  // query token i sees keys [0, L - Sq + i] instead of [0, L)
    int32_t len_add; // tokens appended by this call: sequence b has seq_lens[b] + len_add keys
    const float* k_scale;  // FP8 pools: dequantisation factor per KV head (null = 1)
    const float* v_scale;
    int32_t page_size, bt_stride, num_pages;
    int32_t page_shift;  // log2(page_size) when it is a power of two, else -1
    int64_t cap_tokens;  // bt_stride * page_size (clamp for seq_lens)
    float scale_log2;    // scale * log2(e)
    int32_t min_chunks;
    int32_t spec_chunks;     // chunks per warp prefetched into L2 before griddepcontrol.wait
    int64_t spec_min_total;  // ... only when the call has at least this many chunks in all
    int32_t debug_spec_skew; // test hook: added to every length the speculative pass reads
    int32_t debug_stuck;     // test hook: n > 0 makes CTA 0 / warp n-1's first stage expect 16 bytes too many
    uint64_t wait_limit_ns;  // bound on every mbarrier wait
};

/* Per-warp record of a unit cut by a slice boundary (shared memory, after streaming),
 * kept in the MMA accumulator layout: o[mt][lane] holds that lane's four O^T values of
 * M tile mt, (d, hA) (d, hB) (d+8, hA) (d+8, hB) with d = 16 mt + lane/4,
 * hA = 2 (lane%4), hB = hA + 1.  Global records use the same layout. */
struct __align__(16) Stash {
    float4 o[8][32];  // normalised O^T fragments
    float lse[8];     // log2-sum-exp per head
};

struct Cursor {
    int32_t b, j, c, n, L;  // sequence, unit-in-sequence, chunk-in-unit, chunks, length
};

__device__ __forceinline__ int32_t clamp_len(int64_t L, int64_t cap) {
    if (L < 0) return 0;
    if (L > cap) return (int32_t)cap;
    return (int32_t)L;
}

/* Keys of sequence b: its entry in seq_lens plus the tokens appended by this call. */
__device__ __forceinline__ int64_t keys_of(const DecodeParams& p, int32_t b) {
    return (int64_t)__ldg(p.seq_lens + b) + p.len_add;
}

/* Largest b with pre[b]*U <= x  (x < pre[B]*U). */
__device__ __forceinline__ int32_t find_seq(const uint32_t* pre, int32_t B, int64_t U, int64_t x) {
    int32_t lo = 0, hi = B;
    while (hi - lo > 1) {
        const int32_t mid = (lo + hi) >> 1;
        if ((int64_t)pre[mid] * U <= x) lo = mid; else hi = mid;
    }
    return lo;
}

/* Cursor of flat chunk x from the prefix table alone (L left 0: no global read). */
__device__ __forceinline__ Cursor locate_chunk(const DecodeParams& p, const uint32_t* pre, int64_t x) {
    Cursor cu;
    cu.b = find_seq(pre, p.B, p.U, x);
    cu.n = (int32_t)(pre[cu.b + 1] - pre[cu.b]);
    const int64_t r = x - (int64_t)pre[cu.b] * p.U;
    cu.j = (r <= kSmallProduct) ? (int32_t)((uint32_t)r / (uint32_t)cu.n) : (int32_t)(r / cu.n);
    cu.c = (int32_t)(r - (int64_t)cu.j * cu.n);
    cu.L = 0;
    return cu;
}

__device__ __forceinline__ Cursor locate(const DecodeParams& p, const uint32_t* pre, int64_t x) {
    Cursor cu = locate_chunk(p, pre, x);
    cu.L = clamp_len(keys_of(p, cu.b), p.cap_tokens);
    return cu;
}

/* Page index of token offset t inside a sequence (a shift when P is a power of two). */
__device__ __forceinline__ int32_t page_of(const DecodeParams& p, int32_t t) {
    return p.page_shift >= 0 ? (t >> p.page_shift) : t / p.page_size;
}

/* Step to the next chunk.  Must only be called when a next chunk exists. */
__device__ __forceinline__ void advance(const DecodeParams& p, const uint32_t* pre, Cursor& cu) {
    if (++cu.c < cu.n) return;
    cu.c = 0;
    if (++cu.j < p.U) return;
    cu.j = 0;
    do { ++cu.b; } while (pre[cu.b + 1] == pre[cu.b]);
    cu.n = (int32_t)(pre[cu.b + 1] - pre[cu.b]);
    cu.L = clamp_len(keys_of(p, cu.b), p.cap_tokens);
}

__device__ __forceinline__ int64_t unit_begin(const DecodeParams& p, const uint32_t* pre, int32_t b,
                                              int32_t j) {
    return (int64_t)pre[b] * p.U + (int64_t)j * (pre[b + 1] - pre[b]);
}

/* Writes M tile mt of an O^T fragment as bf16 output rows: movmatrix turns the lane's
 * (d, head pair) values into (head = lane/4, d pair) so each lane stores 2 x 32 bits of
 * the row of head lane/4 (`head_row`).  Collective over the warp; only lanes with
 * `valid` store. */
__device__ __forceinline__ void store_out_tile(__nv_bfloat16* head_row, float f0, float f1, float f2,
                                               float f3, float sA, float sB, int mt, int tig,
                                               bool valid) {
    const uint32_t y0 = ptx::movmatrix_t(ptx::pack_bf16x2(f0 * sA, f1 * sB));
    const uint32_t y1 = ptx::movmatrix_t(ptx::pack_bf16x2(f2 * sA, f3 * sB));
    if (valid) {
        *reinterpret_cast<uint32_t*>(head_row + mt * 16 + 2 * tig) = y0;
        *reinterpret_cast<uint32_t*>(head_row + mt * 16 + 8 + 2 * tig) = y1;
    }
}

/* FP8 pools: the PV accumulator rows of M tile u map to d = 16u + 2*gid (row gid) and
 * 16u + 2*gid + 1 (row gid + 8), the order in which the transposed byte-pair loads
 * deliver V.  After the transposes a lane holds d = 16u + 4*tig + {0, 2} (y0) and
 * {1, 3} (y1) of head gid; interleave and store 4 consecutive values. */
__device__ __forceinline__ void store_out_tile_kv8(__nv_bfloat16* head_row, float f0, float f1,
                                                   float f2, float f3, float sA, float sB, int u,
                                                   int tig, bool valid) {
    const uint32_t y0 = ptx::movmatrix_t(ptx::pack_bf16x2(f0 * sA, f1 * sB));
    const uint32_t y1 = ptx::movmatrix_t(ptx::pack_bf16x2(f2 * sA, f3 * sB));
    if (valid)
        *reinterpret_cast<uint2*>(head_row + u * 16 + 4 * tig) =
            make_uint2(ptx::prmt(y0, y1, 0x5410u), ptx::prmt(y0, y1, 0x7632u));
}

template <bool KV8>
__device__ __forceinline__ void store_tile(__nv_bfloat16* head_row, float f0, float f1, float f2,
                                           float f3, float sA, float sB, int mt, int tig,
                                           bool valid) {
    if (KV8) store_out_tile_kv8(head_row, f0, f1, f2, f3, sA, sB, mt, tig, valid);
    else store_out_tile(head_row, f0, f1, f2, f3, sA, sB, mt, tig, valid);
}

/* Query row r (of the Hq/Hkv * Sq rows of KV head kvh) of sequence b: head kvh*g + r/Sq,
 * token r%Sq.  Returns its offset (in elements) in q / out, whose layout is
 * [B, Sq, Hq, 128]. */
template <bool MQ>
__device__ __forceinline__ int64_t row_offset(const DecodeParams& p, int32_t b, int32_t kvh, int r) {
    if (!MQ) return ((int64_t)b * p.Hq + kvh * p.g + r) * kHeadDim;  // Sq == 1
    const int h = r / p.Sq;
    const int i = r - h * p.Sq;
    return (((int64_t)b * p.Sq + i) * p.Hq + kvh * p.g + h) * kHeadDim;
}

/* Index of query row r of KV head kvh, sequence b, in the [B, Hq, Sq] log-sum-exp output. */
template <bool MQ>
__device__ __forceinline__ int64_t lse_index(const DecodeParams& p, int32_t b, int32_t kvh, int r) {
    if (!MQ) return (int64_t)b * p.Hq + kvh * p.g + r;  // Sq == 1
    const int h = r / p.Sq;
    const int i = r - h * p.Sq;
    return ((int64_t)b * p.Hq + kvh * p.g + h) * p.Sq + i;
}

/* Writes the natural-log sum-exp of this lane's two rows 2tig, 2tig+1 of row group hg
 * from their log2-domain values (lanes with gid == 0 call it; rows past nhv are padding). */
template <bool MQ>
__device__ __forceinline__ void store_lse(const DecodeParams& p, int32_t b, int32_t kvh, int hg,
                                          int nhv, int tig, float lse2A, float lse2B) {
    constexpr float kLn2 = 0.6931471805599453f;
    const int r = 2 * tig;
    if (r < nhv) p.lse_out[lse_index<MQ>(p, b, kvh, hg * kHeadsPerGroup + r)] = lse2A * kLn2;
    if (r + 1 < nhv) p.lse_out[lse_index<MQ>(p, b, kvh, hg * kHeadsPerGroup + r + 1)] = lse2B * kLn2;
}

/* Keys visible to query row r of a sequence of length L. */
template <bool MQ>
__device__ __forceinline__ int32_t row_limit(const DecodeParams& p, int r, int32_t L) {
    if (!MQ || !p.causal || r >= p.rows) return L;
    return L - p.Sq + (r - (r / p.Sq) * p.Sq) + 1;
}

/* Log-sum-exp merge of one head pair of a fragment tile.  Contributions arrive in
 * batches: each batch's maximum is taken first, so the weights of a batch are
 * independent exponentials (no serial rescale chain per contribution). */
template <bool MQ>
struct PairMerge {
    float mA, mB, dA, dB;
    float a0, a1, a2, a3;
    __device__ __forceinline__ void init() {
        mA = mB = -INFINITY;
        dA = dB = 0.f;
        a0 = a1 = a2 = a3 = 0.f;
    }
    /* Raise the running maxima to (bA, bB), rescaling what was accumulated. */
    __device__ __forceinline__ void rebase(float bA, float bB) {
        if (bA > mA) {
            const float s = ptx::ex2(mA - bA);
            dA *= s; a0 *= s; a2 *= s; mA = bA;
        }
        if (bB > mB) {
            const float s = ptx::ex2(mB - bB);
            dB *= s; a1 *= s; a3 *= s; mB = bB;
        }
    }
    /* Add one contribution; its lse must not exceed the current maxima.  A row whose
     * contributions are all empty (lse = -inf; only with several query tokens) keeps
     * weight 0. */
    __device__ __forceinline__ void add(float lseA, float lseB, float4 v) {
        const float wA = ptx::ex2(lseA - ((MQ && mA == -INFINITY) ? 0.f : mA));
        const float wB = ptx::ex2(lseB - ((MQ && mB == -INFINITY) ? 0.f : mB));
        dA += wA; dB += wB;
        a0 = fmaf(wA, v.x, a0); a1 = fmaf(wB, v.y, a1);
        a2 = fmaf(wA, v.z, a2); a3 = fmaf(wB, v.w, a3);
    }
};

/* MQ = false: one query token per sequence (rows = heads, every row sees [0, L)); the
 * per-row masks and empty-row guards compile away.  MQ = true: seqlen_q tokens, optional
 * causal limits per row.
 * KV8 = false: bf16 pools, 8 KB stages (K and V as two 64-dim boxes each), bf16 MMAs.
 * KV8 = true: e4m3 pools, 4 KB stages (one 128-byte box each for K and V); the fp8
 * bytes are converted exactly to f16 after ldmatrix and multiplied with f16 MMAs
 * (q rounded to f16 after an exact per-row power-of-two rescale; P in f16). */
template <int W, int S, bool MQ, bool KV8, int NG, bool LSE>
__global__ void __launch_bounds__(W * 32, 1)
pgqa_decode_kernel(const __grid_constant__ CUtensorMap kmap,
                   const __grid_constant__ CUtensorMap vmap, const DecodeParams p) {
    constexpr int NT = W * 32;
    constexpr int kStage = KV8 ? kStageBytesKv8 : kStageBytes;
    constexpr int kVOff = KV8 ? kHalfBytes : 2 * kHalfBytes;  // V's offset inside a stage
    // A warp's first cut unit goes straight to its own shared-memory slots when it
    // completes (FP8: frees 32 registers; NG > 1: its NG states would not fit in
    // registers); bf16 with NG = 1 keeps it in registers.
    constexpr bool kEarlyStash = KV8 || NG > 1;
    constexpr int kStates = 2 * NG;           // parked states per warp (first, last) x groups
    constexpr int kMiscInts = 32 + 2 * W * kStates;  // warp sums [32] + parked keys int2
    static_assert((kEarlyStash ? NG : 2) * sizeof(Stash) <= (size_t)S * kStage,
                  "the states a warp parks in its ring must fit in it");
    static_assert(W * kStates <= 32, "parked states are scanned one per lane");
    static_assert(W <= 16, "per-warp scan words live in misc[0, 32)");
    extern __shared__ uint8_t smem_raw[];
    // 128-byte TMA swizzle needs 1024-byte aligned stages (shared-window offset).
    uint8_t* smem = smem_raw + ((1024u - (ptx::smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* ring = smem;                                                  // W*S stages
    uint64_t* bars = reinterpret_cast<uint64_t*>(ring + W * S * kStage);   // W*S
    int32_t* misc = reinterpret_cast<int32_t*>(bars + W * S);               // kMiscInts
    uint32_t* pre = reinterpret_cast<uint32_t*>(misc + kMiscInts);          // B+1
    // early stash slots (kEarlyStash): W x NG Stash after the prefix table, 16-byte aligned
    const uint32_t early_base = (ptx::smem_u32(pre + p.B + 1) + 15u) & ~15u;

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int gid = lane >> 2;  // MMA group id (row within an 8-row block)
    const int tig = lane & 3;   // thread in group

    const uint64_t pol = ptx::policy_evict_first();
    if (tid == 0) {
        ptx::prefetch_tensormap(&kmap);
        ptx::prefetch_tensormap(&vmap);
        for (int i = 0; i < W * S; ++i) ptx::mbar_init(ptx::smem_u32(bars + i), 1);
        ptx::fence_mbar_init();
    }

    /* ---- chunk prefix over sequences: pre[b] = chunks before sequence b, pre[B] = all ----
     * (every CTA computes it; B is small).  Thread tid owns sequences [sb0, sb1). */
    const int per_thread = (p.B + NT - 1) / NT;
    const int sb0 = min(p.B, tid * per_thread);
    const int sb1 = min(p.B, sb0 + per_thread);
    auto scan_prefix = [&](auto load_len) {
        uint32_t local = 0, cmin = 0xffffffffu, cmax = 0;
        for (int b = sb0; b < sb1; ++b) {
            const uint32_t nb = (uint32_t)seq_chunks((int64_t)load_len(b) + p.len_add, p.cap_tokens);
            local += nb;
            cmin = min(cmin, nb);
            cmax = max(cmax, nb);
        }
        uint32_t incl = local;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t v = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += v;
        }
        cmin = __reduce_min_sync(0xffffffffu, cmin);
        cmax = __reduce_max_sync(0xffffffffu, cmax);
        if (lane == 31) {
            misc[warp] = (int32_t)incl;
            // the warp's common chunk count; -1: its sequences differ; -2: it has none
            misc[16 + warp] = cmin > cmax ? -2 : (cmin == cmax ? (int32_t)cmin : -1);
        }
        __syncthreads();
        uint32_t run = incl - local;
        for (int w2 = 0; w2 < warp; ++w2) run += (uint32_t)misc[w2];

        if (tid == NT - 1) pre[p.B] = run + local;
        for (int b = sb0; b < sb1; ++b) {
            pre[b] = run;
            run += (uint32_t)seq_chunks((int64_t)load_len(b) + p.len_add, p.cap_tokens);
        }
        __syncthreads();
    };

    /* ---- speculative pass, while the previous grid finishes on other SMs ----
     * (Run only when spec_chunks > 0: the host enables it for calls whose warps stream
     * enough chunks to repay it when no grid is ahead.)
     * The prefix table and the partition are computed from a first read of the lengths
     * and the block table, and each warp prefetches its first chunks into L2.  Only L2
     * sees these reads (ld.global.cg and tensor prefetches; L2 is coherent with the
     * previous grid's writes).  After griddepcontrol.wait every length is read again and
     * the table is kept only if every sequence still has the chunk count it was built
     * from (else it is rebuilt); the block table is read again too, so a predecessor
     * that writes lengths or table only makes the prefetch miss.  Table entries are read
     * only below ceil(L/P) of the clamped length (inside every row by the table's
     * contract) and page ids outside [0, num_pages) are not prefetched. */
    // the warp's first block-table window as the pass located it (sequence, first page,
    // pages of the sequence; sp_b < 0: none)
    int32_t sp_b = -1, sp_p0 = 0, sp_npg = 0;

    /* The partition of the call from the prefix table: T flat chunks, nct active CTAs,
     * this CTA's slice [cs, ce) over wa active warps, this warp's slice [ws, we) and the
     * cursor of its first chunk (length not read yet).  Computed by the pass before
     * griddepcontrol.wait and kept when the lengths check finds the same chunk counts,
     * else computed after it. */
    int64_t T = 0, nct = 0, cs = 0, ce = 0, ws = 0, we = 0;
    int wa = 0;
    Cursor ic0{};
    auto partition = [&]() {
        T = (int64_t)pre[p.B] * p.U;
        nct = T > 0 ? active_ctas(T, gridDim.x, W, p.min_chunks) : 0;
        if ((int64_t)p.B * p.U <= nct && nct % ((int64_t)p.B * p.U) != 0) {
            // every warp of the scan saw the same non-zero chunk count: equal units
            int32_t u = -2;
            bool same = true;
            for (int w2 = 0; w2 < W; ++w2) {
                const int32_t v = misc[16 + w2];
                if (v == -1 || (v >= 0 && u >= 0 && v != u)) same = false;
                if (v >= 0) u = v;
            }
            nct = align_ctas(nct, (int64_t)p.B * p.U, same && u > 0);
        }
        wa = 0;
        if ((int64_t)blockIdx.x >= nct) return;
        cs = slice_begin(blockIdx.x, nct, T);
        ce = slice_begin(blockIdx.x + 1, nct, T);
        wa = (int)active_warps(ce - cs, W);
        if (warp < wa) {
            ws = cs + slice_begin(warp, wa, ce - cs);
            we = cs + slice_begin(warp + 1, wa, ce - cs);
            ic0 = locate_chunk(p, pre, ws);
        }
    };

    if (p.spec_chunks > 0) {
        scan_prefix([&](int b) { return ptx::ld_cg_s32(p.seq_lens + b) + p.debug_spec_skew; });
        partition();
        // the table may be far longer than the sequences: the prefetch needs real length
        if (warp < wa && T >= p.spec_min_total) {
            const int64_t ntot = we - ws;
            const int64_t npf = ntot < p.spec_chunks ? ntot : p.spec_chunks;
            const int P = p.page_size;
            int32_t b = ic0.b, n = ic0.n, j = ic0.j, c = ic0.c;
            int32_t win_b = -1, win_p0 = 0, win_pid = 0;
            for (int64_t k = 0; k < npf; ++k) {
                const int32_t page = page_of(p, c * kChunkTokens);
                if (b != win_b || page < win_p0 || page >= win_p0 + 32) {
                    win_b = b;
                    win_p0 = page;
                    const int32_t npg = page_of(p, n * kChunkTokens + P - 1);
                    const int32_t pg = page + lane;
                    win_pid = (pg < npg)
                                  ? ptx::ld_cg_s32(p.block_table + (int64_t)b * p.bt_stride + pg)
                                  : -1;
                    if (k == 0) { sp_b = b; sp_p0 = page; sp_npg = npg; }
                }
                const int32_t pid = __shfl_sync(0xffffffffu, win_pid, page - win_p0);
                if (lane == 0 && (uint32_t)pid < (uint32_t)p.num_pages) {
                    const int32_t kvh = (p.n_w == 1) ? j : j / p.n_w;
                    const int32_t z = pid * P + (c * kChunkTokens - page * P);
                    ptx::tma_prefetch_l2_3d(&kmap, 0, kvh, z);
                    ptx::tma_prefetch_l2_3d(&vmap, 0, kvh, z);
                    if (!KV8) {
                        ptx::tma_prefetch_l2_3d(&kmap, 64, kvh, z);
                        ptx::tma_prefetch_l2_3d(&vmap, 64, kvh, z);
                    }
                }
                if (k + 1 < npf && ++c == n) {  // step to the next chunk (one exists)
                    c = 0;
                    if (++j == p.U) {
                        j = 0;
                        do { ++b; } while (pre[b + 1] == pre[b]);
                        n = (int32_t)(pre[b + 1] - pre[b]);
                    }
                }
            }
        }
    }

    // Launched as a programmatic dependent: everything above overlaps the previous
    // kernel's tail; of what was read before this point only the prefix table, once
    // checked, and the partition computed from it are used after it.
    ptx::griddep_wait();

    // The warp's first window is read again now (the pass's values may be stale), in the
    // same round trip as the lengths check; it is used when the partition is unchanged,
    // so the first tiles wait for no further load.
    int32_t sp_pid = 0;
    if (sp_b >= 0) {
        const int32_t pg = sp_p0 + lane;
        sp_pid = (pg < sp_npg) ? __ldg(p.block_table + (int64_t)sp_b * p.bt_stride + pg) : 0;
    }
    bool rebuild = true;
    {
        int32_t bad = 0;
        if (p.spec_chunks > 0) {
            int32_t changed = 0;
            for (int b = sb0; b < sb1; ++b) {
                const int32_t L0 = __ldg(p.seq_lens + b);
                const int64_t L = (int64_t)L0 + p.len_add;
                if (L0 < 0 || L > p.cap_tokens) bad = 1;
                if ((uint32_t)seq_chunks(L, p.cap_tokens) != pre[b + 1] - pre[b]) changed = 1;
            }
            rebuild = __syncthreads_or(changed) != 0;
        }
        if (rebuild) {
            scan_prefix([&](int b) {
                const int32_t L0 = __ldg(p.seq_lens + b);
                if (L0 < 0 || (int64_t)L0 + p.len_add > p.cap_tokens) bad = 1;
                return L0;
            });
        }
        if (bad && blockIdx.x == 0) atomicOr(p.err, kErrBadSeqlen);
    }
    if (rebuild) partition();

    /* Zero-length sequences produce zeros (softmax over an empty set) and a log-sum-exp of
     * -inf, written by CTA 0. */
    if (blockIdx.x == 0) {
        for (int b = tid; b < p.B; b += NT) {
            if (pre[b + 1] == pre[b]) {
                uint4* o4 = reinterpret_cast<uint4*>(p.out + (int64_t)b * p.Sq * p.Hq * kHeadDim);
                for (int i = 0; i < p.Sq * p.Hq * kHeadDim / 8; ++i) o4[i] = make_uint4(0, 0, 0, 0);
                if (LSE)
                    for (int i = 0; i < p.Hq * p.Sq; ++i) p.lse_out[(int64_t)b * p.Hq * p.Sq + i] = -INFINITY;
            }
        }
    }

    if (T == 0) return;
    if ((int64_t)blockIdx.x >= nct) return;

    const uint32_t ring_base = ptx::smem_u32(ring);
    const uint32_t bar_base = ptx::smem_u32(bars);

    /* Per-warp streaming state kept until the CTA-level merge (per row group grp). */
    bool have_first = false, have_last = false;
    Cursor first_u{}, last_u{};
    float fo[8][4];                 // first cut unit (NG = 1, bf16 only)
    float flse[2] = {0.f, 0.f};
    float o[NG][8][4];
    float m2[NG][2], l2[NG][2];
    bool aborted = false;

    if (warp < wa) {
        const int64_t ntot = we - ws;

        Cursor ic = ic0;
        ic.L = clamp_len(keys_of(p, ic.b), p.cap_tokens);  // first needed after the first issues
        Cursor cc = ic;

        int32_t win_b = -1, win_p0 = 0, win_pid = 0;
        int64_t issued = 0;
        const int P = p.page_size;
        // page / slot of the issue cursor's chunk and its KV head, stepped with the cursor
        // (no division per chunk: chunks are 16-token aligned and P is a multiple of 16)
        int32_t ipage = page_of(p, ic.c * kChunkTokens);
        int32_t ioff = ic.c * kChunkTokens - ipage * P;
        int32_t ikvh = (p.n_w == 1) ? ic.j : ic.j / p.n_w;
        if (!rebuild && ic.b == sp_b && ipage == sp_p0) {  // the window read after the wait
            win_b = sp_b;
            win_p0 = sp_p0;
            win_pid = sp_pid;
        }

        auto issue_next = [&]() {
            const int32_t page = ipage;
            if (ic.b != win_b || page < win_p0 || page >= win_p0 + 32) {
                win_b = ic.b;
                win_p0 = page;
                // pages of the sequence, ceil(L / P) = ceil(16 n / P) as P is a multiple
                // of 16 (from the chunk count, so the window does not wait for L)
                const int32_t npg = page_of(p, ic.n * kChunkTokens + P - 1);
                const int32_t pg = page + lane;
                win_pid = (pg < npg) ? __ldg(p.block_table + (int64_t)ic.b * p.bt_stride + pg) : 0;
            }
            int32_t pid = __shfl_sync(0xffffffffu, win_pid, page - win_p0);
            if (lane == 0) {
                if ((uint32_t)pid >= (uint32_t)p.num_pages) {
                    atomicOr(p.err, kErrBadPage);
                    pid = 0;
                }
                const int stage = (int)(issued % S);
                const uint32_t bar = bar_base + (uint32_t)(warp * S + stage) * 8u;
                const uint32_t dst = ring_base + (uint32_t)(warp * S + stage) * kStage;
                const int32_t kvh = ikvh;
                const int32_t z = pid * P + ioff;
                const uint32_t extra =
                    (p.debug_stuck == warp + 1 && blockIdx.x == 0 && issued == 0) ? 16u : 0u;
                ptx::mbar_arrive_expect_tx(bar, kStage + extra);
                if (KV8) {
                    ptx::tma_load_3d(dst, &kmap, bar, 0, kvh, z, pol);
                    ptx::tma_load_3d(dst + kVOff, &vmap, bar, 0, kvh, z, pol);
                } else {
                    ptx::tma_load_3d(dst, &kmap, bar, 0, kvh, z, pol);
                    ptx::tma_load_3d(dst + kHalfBytes, &kmap, bar, 64, kvh, z, pol);
                    ptx::tma_load_3d(dst + 2 * kHalfBytes, &vmap, bar, 0, kvh, z, pol);
                    ptx::tma_load_3d(dst + 3 * kHalfBytes, &vmap, bar, 64, kvh, z, pol);
                }
            }
            ++issued;
            if (issued < ntot) {
                advance(p, pre, ic);
                if (ic.c == 0) {  // a new unit starts at its first chunk
                    ipage = 0;
                    ioff = 0;
                    ikvh = (p.n_w == 1) ? ic.j : ic.j / p.n_w;
                } else if ((ioff += kChunkTokens) == P) {
                    ioff = 0;
                    ++ipage;
                }
            }
        };

        const int64_t prologue = ntot < S ? ntot : S;
        for (int64_t k = 0; k < prologue; ++k) issue_next();

        uint32_t qf[NG][16];
        int nh_valid[NG];       // valid rows of each row group (<= 0: an empty group)
        int32_t limA[NG], limB[NG];  // keys visible to this lane's two columns (rows)
        // score multipliers of this lane's two columns and the V factor (FP8 pools)
        float mulA[NG], mulB[NG], vsc = 1.f;
#pragma unroll
        for (int gr = 0; gr < NG; ++gr) { mulA[gr] = p.scale_log2; mulB[gr] = p.scale_log2; }
        auto load_q = [&](const Cursor& cu) {
            const int32_t kvh = cu.j / p.n_w;
            const int32_t wg = cu.j - kvh * p.n_w;
            if (KV8) {
                const float ks = p.k_scale ? __ldg(p.k_scale + kvh) : 1.f;
                vsc = p.v_scale ? __ldg(p.v_scale + kvh) : 1.f;
#pragma unroll
                for (int gr = 0; gr < NG; ++gr) { mulA[gr] = p.scale_log2 * ks; mulB[gr] = mulA[gr]; }
            }
#pragma unroll
            for (int gr = 0; gr < NG; ++gr) {
            const int32_t hg = wg * NG + gr;
            nh_valid[gr] = min(kHeadsPerGroup, p.rows - hg * kHeadsPerGroup);
            limA[gr] = row_limit<MQ>(p, hg * kHeadsPerGroup + 2 * tig, cu.L);
            limB[gr] = row_limit<MQ>(p, hg * kHeadsPerGroup + 2 * tig + 1, cu.L);
            if (KV8) {
                /* qf[gr][4m + 2hh + j] = f16 pair q[32m + 16hh + 4tig + 2j + {0,1}] of row
                 * gid, the d order of the converted K fragments.  The row is scaled by 2^e
                 * (exact) so that its largest |q| lies in [2^14, 2^15): f16 then keeps all
                 * of bf16's precision without overflow; 2^-e goes into the score
                 * multiplier of that column. */
                float qv[32];
                if (gid < nh_valid[gr]) {
                    const __nv_bfloat16* qp = p.q + row_offset<MQ>(p, cu.b, kvh, hg * kHeadsPerGroup + gid);
#pragma unroll
                    for (int k = 0; k < 8; ++k) {
                        const uint2 w = __ldg(reinterpret_cast<const uint2*>(qp + 16 * k + 4 * tig));
                        const float2 f0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w.x));
                        const float2 f1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w.y));
                        qv[4 * k] = f0.x; qv[4 * k + 1] = f0.y; qv[4 * k + 2] = f1.x; qv[4 * k + 3] = f1.y;
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < 32; ++i) qv[i] = 0.f;
                }
                float mx = 0.f;
#pragma unroll
                for (int i = 0; i < 32; ++i) mx = fmaxf(mx, fabsf(qv[i]));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
                int e = 0;
                if (mx > 0.f) e = 14 - ((int)((__float_as_uint(mx) >> 23) & 0xff) - 127);
                e = max(-126, min(60, e));
                const float up = __uint_as_float((uint32_t)(e + 127) << 23);
                const float down = __uint_as_float((uint32_t)(127 - e) << 23);
#pragma unroll
                for (int i = 0; i < 16; ++i) qf[gr][i] = ptx::pack_f16x2(qv[2 * i] * up, qv[2 * i + 1] * up);
                mulA[gr] *= __shfl_sync(0xffffffffu, down, 8 * tig);
                mulB[gr] *= __shfl_sync(0xffffffffu, down, 8 * tig + 4);
            } else if (gid < nh_valid[gr]) {
                const uint32_t* qp = reinterpret_cast<const uint32_t*>(
                    p.q + row_offset<MQ>(p, cu.b, kvh, hg * kHeadsPerGroup + gid));
#pragma unroll
                for (int ks = 0; ks < 8; ++ks) {
                    qf[gr][2 * ks] = __ldg(qp + 8 * ks + tig);
                    qf[gr][2 * ks + 1] = __ldg(qp + 8 * ks + 4 + tig);
                }
            } else {
#pragma unroll
                for (int i = 0; i < 16; ++i) qf[gr][i] = 0u;
            }
            }
        };
        auto reset_state = [&]() {
#pragma unroll
            for (int gr = 0; gr < NG; ++gr) {
                m2[gr][0] = m2[gr][1] = -INFINITY;
                l2[gr][0] = l2[gr][1] = 0.f;
#pragma unroll
                for (int mt = 0; mt < 8; ++mt) o[gr][mt][0] = o[gr][mt][1] = o[gr][mt][2] = o[gr][mt][3] = 0.f;
            }
        };

        load_q(cc);
        reset_state();
        bool unit_start_seen = (cc.c == 0);
        int units_done = 0;

        /* Per-lane ldmatrix offsets inside a stage (128-byte swizzle: 16-byte chunk
         * index XOR (row & 7)). */
        const int mj = lane >> 3;  // which 8x8 matrix this lane addresses
        const int mr = lane & 7;   // row within that matrix
        const int tK = mr + 8 * (mj & 1);
        const int tV = mr + 8 * (mj >> 1);

        /* One step streams NC = 1 chunk, or NC = 2 consecutive chunks of the same unit
         * (FP8 pools: two independent QK chains and one softmax vote per 32 tokens; the
         * 4-stage ring keeps two more chunks in flight meanwhile).  Returns false when a
         * wait expired (the ring is drained and the warp stops). */
        constexpr bool kPair = KV8;
        int64_t i = 0;
        auto step = [&](auto nc_tag) -> bool {
            constexpr int NC = decltype(nc_tag)::value;
#pragma unroll
            for (int c = 0; c < NC; ++c) {
                const int64_t k = i + c;
                const uint32_t bar = bar_base + (uint32_t)(warp * S + (int)(k % S)) * 8u;
                if (!ptx::wait_parity_bounded(bar, (uint32_t)((k / S) & 1), p.wait_limit_ns)) {
                    if (lane == 0) atomicOr(p.err, kErrTimeout);
                    aborted = true;
                    // Drain: wait (bounded) for every copy still in flight into this ring.
                    for (int64_t k2 = k; k2 < issued; ++k2) {
                        const uint32_t b2 = bar_base + (uint32_t)(warp * S + (int)(k2 % S)) * 8u;
                        ptx::wait_parity_bounded(b2, (uint32_t)((k2 / S) & 1), p.wait_limit_ns);
                    }
                    return false;
                }
            }
            // only the step's last chunk can be the last of its unit
            const bool last_of_unit = (cc.c + NC - 1 == cc.n - 1);
            const int nvalid = last_of_unit ? (cc.L - (cc.c + NC - 1) * kChunkTokens) : kChunkTokens;
            if (nvalid < kChunkTokens) {
                /* Tokens past the sequence end inside the last page: zero their V rows so
                 * that p = 0 never meets a non-finite V value (0 * NaN). */
                const int64_t k = i + NC - 1;
                uint8_t* vrow = ring + (size_t)(warp * S + (int)(k % S)) * kStage + kVOff;
                if (KV8) {
                    const int units = (kChunkTokens - nvalid) * 8;  // 16-byte pieces of 128-B rows
                    for (int u = lane; u < units; u += 32)
                        *reinterpret_cast<uint4*>(vrow + (nvalid + (u >> 3)) * 128 + (u & 7) * 16) =
                            make_uint4(0, 0, 0, 0);
                } else {
                    const int units = (kChunkTokens - nvalid) * 16;  // 16-byte pieces, both halves
                    for (int u = lane; u < units; u += 32) {
                        const int t = nvalid + (u >> 4);
                        const int half = (u >> 3) & 1;
                        const int c16 = u & 7;
                        *reinterpret_cast<uint4*>(vrow + half * kHalfBytes + t * 128 + c16 * 16) =
                            make_uint4(0, 0, 0, 0);
                    }
                }
                ptx::fence_proxy_async_smem();  // before TMA overwrites this stage again
                __syncwarp();
            }

            /* ---- S^T = K . Q^T : 16 tokens x 8 query rows per chunk and group, K-dim 128 ----
             * s[c][gr][0]: (t=gid, h=2tig) [1]: (gid, 2tig+1) [2]: (gid+8, 2tig)
             * [3]: (gid+8, 2tig+1); every K fragment serves the NG row groups. */
            float s[NC][NG][4];
#pragma unroll
            for (int c = 0; c < NC; ++c) {
                const uint32_t sK = ring_base + (uint32_t)(warp * S + (int)((i + c) % S)) * kStage;
                float sa[NG][4], sb[NG][4];
#pragma unroll
                for (int gr = 0; gr < NG; ++gr)
#pragma unroll
                    for (int r = 0; r < 4; ++r) sa[gr][r] = sb[gr][r] = 0.f;
                if (KV8) {
                    /* One ldmatrix.x4 per 32 dims: matrices (t 0-7 | 8-15) x (16-byte units
                     * 2m | 2m+1); a lane gets 4 consecutive fp8 of one token, which convert
                     * exactly into the A fragments of two k16 f16 MMAs (k slot 2tig+j <-> d
                     * 4tig+j, 2tig+8+j <-> 4tig+2+j, matched by qf's order).  (e4m3 MMAs on
                     * the stored bytes, with q split in two e4m3 parts, measured slower.) */
#pragma unroll
                    for (int m = 0; m < 4; ++m) {
                        const int u = 2 * m + (mj >> 1);
                        const uint32_t addr = sK + tK * 128 + ((u ^ mr) << 4);
                        uint32_t r0, r1, r2, r3;
                        ptx::ldsm_x4(addr, r0, r1, r2, r3);
                        uint32_t k0l, k0h, k1l, k1h, k2l, k2h, k3l, k3h;
                        ptx::e4m3x4_to_f16(r0, k0l, k0h);
                        ptx::e4m3x4_to_f16(r1, k1l, k1h);
                        ptx::e4m3x4_to_f16(r2, k2l, k2h);
                        ptx::e4m3x4_to_f16(r3, k3l, k3h);
#pragma unroll
                        for (int gr = 0; gr < NG; ++gr) {
                            ptx::mma_f16_16816(sa[gr], k0l, k1l, k0h, k1h, qf[gr][4 * m], qf[gr][4 * m + 1]);
                            ptx::mma_f16_16816(sb[gr], k2l, k3l, k2h, k3h, qf[gr][4 * m + 2], qf[gr][4 * m + 3]);
                        }
                    }
#pragma unroll
                    for (int gr = 0; gr < NG; ++gr) {
                        s[c][gr][0] = (sa[gr][0] + sb[gr][0]) * mulA[gr];
                        s[c][gr][1] = (sa[gr][1] + sb[gr][1]) * mulB[gr];
                        s[c][gr][2] = (sa[gr][2] + sb[gr][2]) * mulA[gr];
                        s[c][gr][3] = (sa[gr][3] + sb[gr][3]) * mulB[gr];
                    }
                } else {
#pragma unroll
                    for (int ks = 0; ks < 8; ++ks) {
                        const int half = ks >> 2;
                        const int ch = ((2 * ks) + (mj >> 1)) & 7;
                        const uint32_t addr = sK + half * kHalfBytes + tK * 128 + ((ch ^ mr) << 4);
                        uint32_t a0, a1, a2, a3;
                        ptx::ldsm_x4(addr, a0, a1, a2, a3);
#pragma unroll
                        for (int gr = 0; gr < NG; ++gr) {
                            if (ks & 1) ptx::mma_bf16_16816(sb[gr], a0, a1, a2, a3, qf[gr][2 * ks], qf[gr][2 * ks + 1]);
                            else        ptx::mma_bf16_16816(sa[gr], a0, a1, a2, a3, qf[gr][2 * ks], qf[gr][2 * ks + 1]);
                        }
                    }
#pragma unroll
                    for (int gr = 0; gr < NG; ++gr)
#pragma unroll
                        for (int r = 0; r < 4; ++r) s[c][gr][r] = (sa[gr][r] + sb[gr][r]) * p.scale_log2;
                }
#pragma unroll
                for (int gr = 0; gr < NG; ++gr) {
                    if (MQ) {
                        // keys past the row's limit (the sequence end, or the causal bound) -> -inf
                        const int32_t t = (cc.c + c) * kChunkTokens + gid;
                        s[c][gr][0] = (t < limA[gr]) ? s[c][gr][0] : -INFINITY;
                        s[c][gr][1] = (t < limB[gr]) ? s[c][gr][1] : -INFINITY;
                        s[c][gr][2] = (t + 8 < limA[gr]) ? s[c][gr][2] : -INFINITY;
                        s[c][gr][3] = (t + 8 < limB[gr]) ? s[c][gr][3] : -INFINITY;
                    } else if (c == NC - 1 && nvalid < kChunkTokens) {
                        // tokens past the sequence end -> -inf (every row sees the same keys)
                        if (gid >= nvalid) { s[c][gr][0] = -INFINITY; s[c][gr][1] = -INFINITY; }
                        if (gid + 8 >= nvalid) { s[c][gr][2] = -INFINITY; s[c][gr][3] = -INFINITY; }
                    }
                }
            }

            /* ---- online softmax (log2 domain), heads hA = 2tig, hB = 2tig+1 ----
             * Lazy rescale: the reference max m2 of a column moves only when one of its
             * scores exceeds it by more than kLazyLog2, so p <= 2^kLazyLog2 (fine in f16 /
             * bf16 and fp32).  o and l share the reference, so the result is the same; the
             * column reduction and the rescale of o and l run only when a lane votes. */
            float mxA[NG], mxB[NG];
            bool vote = false;
#pragma unroll
            for (int gr = 0; gr < NG; ++gr) {
                mxA[gr] = fmaxf(s[0][gr][0], s[0][gr][2]);
                mxB[gr] = fmaxf(s[0][gr][1], s[0][gr][3]);
#pragma unroll
                for (int c = 1; c < NC; ++c) {
                    mxA[gr] = fmaxf(mxA[gr], fmaxf(s[c][gr][0], s[c][gr][2]));
                    mxB[gr] = fmaxf(mxB[gr], fmaxf(s[c][gr][1], s[c][gr][3]));
                }
                vote = vote || mxA[gr] > m2[gr][0] + kLazyLog2 || mxB[gr] > m2[gr][1] + kLazyLog2;
            }
            if (__any_sync(0xffffffffu, vote)) {
#pragma unroll
                for (int gr = 0; gr < NG; ++gr) {
#pragma unroll
                    for (int off = 4; off < 32; off <<= 1) {
                        mxA[gr] = fmaxf(mxA[gr], __shfl_xor_sync(0xffffffffu, mxA[gr], off));
                        mxB[gr] = fmaxf(mxB[gr], __shfl_xor_sync(0xffffffffu, mxB[gr], off));
                    }
                    const float mnA = fmaxf(m2[gr][0], mxA[gr]);
                    const float mnB = fmaxf(m2[gr][1], mxB[gr]);
                    // a row with no visible key yet keeps max -inf: rescale against 0 instead
                    const float zA = (MQ && mnA == -INFINITY) ? 0.f : mnA;
                    const float zB = (MQ && mnB == -INFINITY) ? 0.f : mnB;
                    const float alA = ptx::ex2(m2[gr][0] - zA);
                    const float alB = ptx::ex2(m2[gr][1] - zB);
                    m2[gr][0] = mnA;
                    m2[gr][1] = mnB;
                    l2[gr][0] *= alA;
                    l2[gr][1] *= alB;
#pragma unroll
                    for (int mt = 0; mt < 8; ++mt) {
                        o[gr][mt][0] *= alA; o[gr][mt][1] *= alB; o[gr][mt][2] *= alA; o[gr][mt][3] *= alB;
                    }
                }
            }
#pragma unroll
            for (int c = 0; c < NC; ++c) {
                uint32_t pb[NG][2];
#pragma unroll
                for (int gr = 0; gr < NG; ++gr) {
                    // (with one query token every chunk holds a visible key for every row)
                    const float bsA = (MQ && m2[gr][0] == -INFINITY) ? 0.f : m2[gr][0];
                    const float bsB = (MQ && m2[gr][1] == -INFINITY) ? 0.f : m2[gr][1];
                    const float p0 = ptx::ex2(s[c][gr][0] - bsA);
                    const float p1 = ptx::ex2(s[c][gr][1] - bsB);
                    const float p2 = ptx::ex2(s[c][gr][2] - bsA);
                    const float p3 = ptx::ex2(s[c][gr][3] - bsB);
                    l2[gr][0] += p0 + p2;
                    l2[gr][1] += p1 + p3;
                    /* P^T (tokens x heads) C-fragment -> B-fragment of the PV MMA. */
                    pb[gr][0] = ptx::movmatrix_t(KV8 ? ptx::pack_f16x2(p0, p1) : ptx::pack_bf16x2(p0, p1));
                    pb[gr][1] = ptx::movmatrix_t(KV8 ? ptx::pack_f16x2(p2, p3) : ptx::pack_bf16x2(p2, p3));
                }

                /* ---- O^T += V^T . P^T : 128 dims (8 M tiles) x 8 rows, K-dim = 16 tokens;
                 * every V fragment serves the NG row groups ---- */
                const uint32_t sV = ring_base + (uint32_t)(warp * S + (int)((i + c) % S)) * kStage + kVOff;
                if (KV8) {
                    /* ldmatrix.trans on byte pairs: a lane gets V[2tig][d0], V[2tig][d0+1],
                     * V[2tig+1][d0], V[2tig+1][d0+1] (d0 = 16u + 2gid); one byte permute
                     * makes token pairs, converted to the A fragment whose rows gid / gid+8
                     * are d0 / d0+1 (store_out_tile_kv8 undoes that order). */
#pragma unroll
                    for (int c2 = 0; c2 < 4; ++c2) {
                        const int u = 2 * c2 + (mj >> 1);
                        const uint32_t addr = sV + tK * 128 + ((u ^ mr) << 4);
                        uint32_t r[4];
                        ptx::ldsm_x4_t(addr, r[0], r[1], r[2], r[3]);
                        uint32_t x[4], y[4];
#pragma unroll
                        for (int k = 0; k < 4; ++k) ptx::e4m3x4_to_f16(ptx::prmt(r[k], r[k], 0x3120u), x[k], y[k]);
#pragma unroll
                        for (int gr = 0; gr < NG; ++gr) {
                            ptx::mma_f16_16816(o[gr][2 * c2], x[0], y[0], x[1], y[1], pb[gr][0], pb[gr][1]);
                            ptx::mma_f16_16816(o[gr][2 * c2 + 1], x[2], y[2], x[3], y[3], pb[gr][0], pb[gr][1]);
                        }
                    }
                } else {
#pragma unroll
                    for (int mt = 0; mt < 8; ++mt) {
                        const int half = mt >> 2;
                        const int ch = ((2 * mt) + (mj & 1)) & 7;
                        const uint32_t addr = sV + half * kHalfBytes + tV * 128 + ((ch ^ mr) << 4);
                        uint32_t a0, a1, a2, a3;
                        ptx::ldsm_x4_t(addr, a0, a1, a2, a3);
#pragma unroll
                        for (int gr = 0; gr < NG; ++gr)
                            ptx::mma_bf16_16816(o[gr][mt], a0, a1, a2, a3, pb[gr][0], pb[gr][1]);
                    }
                }
            }
            __syncwarp();
#pragma unroll
            for (int c = 0; c < NC; ++c)
                if (issued < ntot) issue_next();  // refills the stages just consumed

            cc.c += NC - 1;  // the cursor now names the step's last chunk
            const bool last_of_warp = (i + NC - 1 == ntot - 1);
            if (last_of_unit || last_of_warp) {
                /* ---- finish this warp's part of the unit, one row group at a time ---- */
                const bool full = unit_start_seen && last_of_unit;
#pragma unroll
                for (int gr = 0; gr < NG; ++gr) {
                    float lA = l2[gr][0], lB = l2[gr][1];
#pragma unroll
                    for (int off = 4; off < 32; off <<= 1) {
                        lA += __shfl_xor_sync(0xffffffffu, lA, off);
                        lB += __shfl_xor_sync(0xffffffffu, lB, off);
                    }
                    // a row with no visible key gives 0 (only with several query tokens);
                    // FP8 pools fold V's dequantisation factor in here
                    const float invA = (!MQ || lA > 0.f) ? (KV8 ? vsc : 1.f) / lA : 0.f;
                    const float invB = (!MQ || lB > 0.f) ? (KV8 ? vsc : 1.f) / lB : 0.f;
                    if (full) {
                        if (nh_valid[gr] > 0) {  // an empty group (rows past g * Sq) stores nothing
                            const int32_t kvh = cc.j / p.n_w;
                            const int32_t hg = (cc.j - kvh * p.n_w) * NG + gr;
                            __nv_bfloat16* orow = p.out + row_offset<MQ>(
                                p, cc.b, kvh, hg * kHeadsPerGroup + min(gid, nh_valid[gr] - 1));
#pragma unroll
                            for (int mt = 0; mt < 8; ++mt)
                                store_tile<KV8>(orow, o[gr][mt][0], o[gr][mt][1], o[gr][mt][2],
                                                o[gr][mt][3], invA, invB, mt, tig, gid < nh_valid[gr]);
                            if (LSE && gid == 0)
                                store_lse<MQ>(p, cc.b, kvh, hg, nh_valid[gr], tig,
                                              m2[gr][0] + ptx::lg2(lA), m2[gr][1] + ptx::lg2(lB));
                        }
                    } else {
                        const float lseA = m2[gr][0] + ptx::lg2(lA);
                        const float lseB = m2[gr][1] + ptx::lg2(lB);
                        if (units_done == 0) {
                            if (kEarlyStash) {
                                const uint32_t a0 = early_base + (uint32_t)((warp * NG + gr) * sizeof(Stash));
#pragma unroll
                                for (int mt = 0; mt < 8; ++mt)
                                    ptx::sts_f4(a0 + (mt * 32 + lane) * 16,
                                                make_float4(o[gr][mt][0] * invA, o[gr][mt][1] * invB,
                                                            o[gr][mt][2] * invA, o[gr][mt][3] * invB));
                                if (gid == 0)
                                    ptx::sts_f2(a0 + offsetof(Stash, lse) + tig * 8, make_float2(lseA, lseB));
                            } else {
#pragma unroll
                                for (int mt = 0; mt < 8; ++mt) {
                                    fo[mt][0] = o[0][mt][0] * invA; fo[mt][1] = o[0][mt][1] * invB;
                                    fo[mt][2] = o[0][mt][2] * invA; fo[mt][3] = o[0][mt][3] * invB;
                                }
                                flse[0] = lseA; flse[1] = lseB;
                            }
                        } else {
                            // Only the warp's last unit can be cut at its end: keep it in place.
#pragma unroll
                            for (int mt = 0; mt < 8; ++mt) {
                                o[gr][mt][0] *= invA; o[gr][mt][1] *= invB;
                                o[gr][mt][2] *= invA; o[gr][mt][3] *= invB;
                            }
                            m2[gr][0] = lseA; m2[gr][1] = lseB;
                        }
                    }
                }
                if (!full) {
                    if (units_done == 0) { first_u = cc; have_first = true; }
                    else { last_u = cc; have_last = true; }
                }
                ++units_done;
                if (!last_of_warp) {
                    advance(p, pre, cc);
                    load_q(cc);
                    reset_state();
                    unit_start_seen = true;
                }
            } else {
                ++cc.c;
            }
            return true;
        };

        while (i < ntot) {
            if (kPair && i + 1 < ntot && cc.c + 1 < cc.n) {
                if (!step(std::integral_constant<int, 2>{})) break;
                i += 2;
            } else {
                if (!step(std::integral_constant<int, 1>{})) break;
                i += 1;
            }
        }

        if (aborted) {
            /* A wait expired and the warp stopped early.  It still parks a state for each
             * unit its slice cuts (the slice's first unit when it starts before the slice
             * or ends after it; its last unit when it ends after the slice), in the slots
             * a complete run would have used, with weight zero (lse = -inf, o = 0).  The
             * CTA then arrives on every arrival counter it owns, the last arriver of each
             * resets it, and the workspace is left zeroed for the next call even though
             * this call's output is not valid (the error word says so). */
            const Cursor u0 = locate(p, pre, ws);
            const Cursor u1 = locate(p, pre, we - 1);
            const bool same = (u0.b == u1.b && u0.j == u1.j);
            have_first = (u0.c != 0) || (same && u1.c != u1.n - 1);
            have_last = !same && (u1.c != u1.n - 1);
            first_u = u0;
            last_u = u1;
#pragma unroll
            for (int gr = 0; gr < NG; ++gr) {
                m2[gr][0] = m2[gr][1] = -INFINITY;
#pragma unroll
                for (int mt = 0; mt < 8; ++mt) o[gr][mt][0] = o[gr][mt][1] = o[gr][mt][2] = o[gr][mt][3] = 0.f;
                if (kEarlyStash && have_first) {
                    const uint32_t a0 = early_base + (uint32_t)((warp * NG + gr) * sizeof(Stash));
#pragma unroll
                    for (int mt = 0; mt < 8; ++mt)
                        ptx::sts_f4(a0 + (mt * 32 + lane) * 16, make_float4(0.f, 0.f, 0.f, 0.f));
                    if (gid == 0)
                        ptx::sts_f2(a0 + offsetof(Stash, lse) + tig * 8, make_float2(-INFINITY, -INFINITY));
                }
            }
#pragma unroll
            for (int mt = 0; mt < 8; ++mt) fo[mt][0] = fo[mt][1] = fo[mt][2] = fo[mt][3] = 0.f;
            flse[0] = flse[1] = -INFINITY;
        }
    }

    // Streaming is over: let the next kernel in the stream start launching (it still
    // waits for this grid's completion before it uses any memory it reads).
    ptx::griddep_launch_dependents();

    /* ---- park this warp's cut units in its own (now idle) ring: no TMA is in flight ----
     * Parked state f = (2 * warp + slot) * NG + grp (slot 0: the warp's first cut unit,
     * 1: its last; grp: row group) lives at the start of warp `warp`'s ring -- slot 0 in
     * the early-stash slots when kEarlyStash.  Its key (b, unit * NG + grp), or (-1, -1)
     * when empty, goes to a compact table for the run scan. */
    auto stash_addr = [&](int f) -> uint32_t {
        const int wf = f / (2 * NG), slot = (f / NG) & 1, gr = f % NG;
        if (kEarlyStash) {  // slot 0 in the early-stash slots, slot 1 at the ring's start
            if (slot == 0) return early_base + (uint32_t)((wf * NG + gr) * sizeof(Stash));
            return ring_base + (uint32_t)(wf * S * kStage + gr * sizeof(Stash));
        }
        return ring_base + (uint32_t)(wf * S * kStage) + (uint32_t)(slot * sizeof(Stash));
    };
    // a row group past g * Sq (the second group of an odd count) has no rows: no state
    auto group_used = [&](const Cursor& cu, int gr) {
        if (NG == 1) return true;  // a unit is one row group, always within the rows
        return ((cu.j % p.n_w) * NG + gr) * kHeadsPerGroup < p.rows;
    };
    const uint32_t keys_base = ptx::smem_u32(misc + 32);  // int2 keys[2 W NG]
    {
        const bool v0 = (warp < wa) && have_first;
        const bool v1 = (warp < wa) && have_last;
        if (v0 && !kEarlyStash) {
            const uint32_t a0 = stash_addr(2 * warp);
#pragma unroll
            for (int mt = 0; mt < 8; ++mt)
                ptx::sts_f4(a0 + (mt * 32 + lane) * 16, make_float4(fo[mt][0], fo[mt][1], fo[mt][2], fo[mt][3]));
            if (gid == 0) ptx::sts_f2(a0 + offsetof(Stash, lse) + tig * 8, make_float2(flse[0], flse[1]));
        }
#pragma unroll
        for (int gr = 0; gr < NG; ++gr) {
            if (v1) {
                const uint32_t a1 = stash_addr((2 * warp + 1) * NG + gr);
#pragma unroll
                for (int mt = 0; mt < 8; ++mt)
                    ptx::sts_f4(a1 + (mt * 32 + lane) * 16,
                                make_float4(o[gr][mt][0], o[gr][mt][1], o[gr][mt][2], o[gr][mt][3]));
                if (gid == 0) ptx::sts_f2(a1 + offsetof(Stash, lse) + tig * 8, make_float2(m2[gr][0], m2[gr][1]));
            }
            if (lane == 0) {
                ptx::sts_i2(keys_base + ((2 * warp) * NG + gr) * 8,
                            v0 && group_used(first_u, gr) ? make_int2(first_u.b, first_u.j * NG + gr)
                                                          : make_int2(-1, -1));
                ptx::sts_i2(keys_base + ((2 * warp + 1) * NG + gr) * 8,
                            v1 && group_used(last_u, gr) ? make_int2(last_u.b, last_u.j * NG + gr)
                                                         : make_int2(-1, -1));
            }
        }
    }
    __syncthreads();

    /* ---- CTA level: merge every cut unit; warp w owns M tiles w, w+W, ... ----
     * Parked states of one unit form a run in (warp, slot) order (slices are contiguous).
     * For each run every warp LSE-merges its M tiles across the run, then either stores
     * the output (unit inside this CTA) or writes that tile of the CTA's record and
     * counts arrivals per (unit, M tile); the warp that completes a tile merges it across
     * all CTAs' records.  Merges take the maximum first and select, never branch, on
     * membership, so every load of a pass is issued at once. */
    constexpr int NF = W * kStates;
    int2 key = make_int2(-1, -1);
    if (lane < NF) key = ptx::lds_i2(keys_base + lane * 8);
    const unsigned vmask = __ballot_sync(0xffffffffu, lane < NF && key.x >= 0);
    unsigned rem = vmask;
    while (rem) {
        const int fa = __ffs(rem) - 1;
        const int32_t ub = __shfl_sync(0xffffffffu, key.x, fa);
        const int32_t uj = __shfl_sync(0xffffffffu, key.y, fa);
        const unsigned run = __ballot_sync(0xffffffffu, ((vmask >> lane) & 1u) && key.x == ub && key.y == uj);
        rem &= ~run;

        const int32_t uu = uj / NG;        // the unit
        const int gq = uj - uu * NG;         // its row group, the same for the whole run
        const int32_t n_u = (int32_t)(pre[ub + 1] - pre[ub]);
        const int64_t ubeg = unit_begin(p, pre, ub, uu);
        const int32_t kvh = uu / p.n_w;
        const int32_t hg = (uu - kvh * p.n_w) * NG + gq;
        const int nhv = min(kHeadsPerGroup, p.rows - hg * kHeadsPerGroup);
        const bool inside = (ubeg >= cs && ubeg + n_u <= ce);
        __nv_bfloat16* orow = p.out + row_offset<MQ>(p, ub, kvh, hg * kHeadsPerGroup + min(gid, nhv - 1));
        // only states of row group gq can be in the run: f = fi * NG + gq
        constexpr int NFG = NF / NG;
        for (int mt = warp; mt < 8; mt += W) {
            float2 ls[NFG];
            float4 v[NFG];
#pragma unroll
            for (int fi = 0; fi < NFG; ++fi) {
                const uint32_t sa = stash_addr(fi * NG + gq);
                ls[fi] = ptx::lds_f2(sa + offsetof(Stash, lse) + tig * 8);
                v[fi] = ptx::lds_f4(sa + (mt * 32 + lane) * 16);
            }
            float bA = -INFINITY, bB = -INFINITY;
#pragma unroll
            for (int fi = 0; fi < NFG; ++fi) {
                const bool in = (run >> (fi * NG + gq)) & 1u;
                bA = in ? fmaxf(bA, ls[fi].x) : bA;
                bB = in ? fmaxf(bB, ls[fi].y) : bB;
            }
            float dA = 0.f, dB = 0.f, a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
            const float zA = (MQ && bA == -INFINITY) ? 0.f : bA;  // rows with no key: weight 0
            const float zB = (MQ && bB == -INFINITY) ? 0.f : bB;
#pragma unroll
            for (int fi = 0; fi < NFG; ++fi) {
                const bool in = (run >> (fi * NG + gq)) & 1u;
                const float wA = ptx::ex2(ls[fi].x - zA), wB = ptx::ex2(ls[fi].y - zB);
                dA = in ? dA + wA : dA;
                dB = in ? dB + wB : dB;
                a0 = in ? fmaf(wA, v[fi].x, a0) : a0;
                a1 = in ? fmaf(wB, v[fi].y, a1) : a1;
                a2 = in ? fmaf(wA, v[fi].z, a2) : a2;
                a3 = in ? fmaf(wB, v[fi].w, a3) : a3;
            }
            const float invA = (!MQ || dA > 0.f) ? 1.f / dA : 0.f;
            const float invB = (!MQ || dB > 0.f) ? 1.f / dB : 0.f;
            if (inside) {
                store_tile<KV8>(orow, a0, a1, a2, a3, invA, invB, mt, tig, gid < nhv);
                if (LSE && mt == 0 && gid == 0)
                    store_lse<MQ>(p, ub, kvh, hg, nhv, tig, bA + ptx::lg2(dA), bB + ptx::lg2(dB));
                continue;
            }
            const int64_t slot = record_slot(blockIdx.x, cs, ubeg) * NG + gq;
            reinterpret_cast<float4*>(p.rec_o)[(slot * 8 + mt) * 32 + lane] =
                make_float4(a0 * invA, a1 * invB, a2 * invA, a3 * invB);
            if (gid == 0)
                reinterpret_cast<float2*>(p.rec_lse)[(slot * 8 + mt) * 4 + tig] =
                    make_float2(bA + ptx::lg2(dA), bB + ptx::lg2(dB));
            const int64_t c_first = slice_owner(ubeg, nct, T);
            const int64_t c_last = slice_owner(ubeg + n_u - 1, nct, T);
            int last = 0;
            __syncwarp();  // the warp's record stores happen before lane 0's release
            if (lane == 0) {
                int32_t* cnt = p.counters + (((int64_t)ub * p.U + uu) * NG + gq) * 8 + mt;
                // releases this CTA's record tile (the warp's stores, ordered before lane 0
                // by the __syncwarp above) and, for the last arriver, acquires the others'
                // (one acq_rel atomic measured faster than fence + relaxed atomic + fence)
                const int32_t prev = ptx::atom_add_acq_rel_gpu(cnt, 1);
                if (prev == (int32_t)(c_last - c_first)) {
                    *cnt = 0;                  // leave the workspace zeroed for the next call
                    last = 1;
                }
            }
            last = __shfl_sync(0xffffffffu, last, 0);
            __syncwarp();
            if (!last) continue;
            // This warp completed tile mt: merge it over every CTA's record, 16 at a time.
            const int nrec = (int)(c_last - c_first + 1);
            // Record slots: CTA c_first holds the unit's head in slot 2c+1 unless its slice
            // starts exactly at the unit; every later CTA holds it in slot 2c.
            const int64_t slot0 = record_slot(c_first, slice_begin(c_first, nct, T), ubeg) * NG + gq;
            PairMerge<MQ> g;
            g.init();
            for (int r0 = 0; r0 < nrec; r0 += 16) {
                float2 lse[16];
                float4 rv[16];
#pragma unroll
                for (int u = 0; u < 16; ++u) {
                    lse[u] = make_float2(-INFINITY, -INFINITY);
                    rv[u] = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (r0 + u < nrec) {
                        const int64_t sl = (r0 + u == 0) ? slot0 : 2 * (c_first + r0 + u) * NG + gq;
                        lse[u] = __ldcg(reinterpret_cast<const float2*>(p.rec_lse) + (sl * 8 + mt) * 4 + tig);
                        rv[u] = __ldcg(reinterpret_cast<const float4*>(p.rec_o) + (sl * 8 + mt) * 32 + lane);
                    }
                }
                float rA = -INFINITY, rB = -INFINITY;
#pragma unroll
                for (int u = 0; u < 16; ++u) { rA = fmaxf(rA, lse[u].x); rB = fmaxf(rB, lse[u].y); }
                g.rebase(rA, rB);
#pragma unroll
                for (int u = 0; u < 16; ++u)
                    if (r0 + u < nrec) g.add(lse[u].x, lse[u].y, rv[u]);
            }
            store_tile<KV8>(orow, g.a0, g.a1, g.a2, g.a3, (!MQ || g.dA > 0.f) ? 1.f / g.dA : 0.f,
                           (!MQ || g.dB > 0.f) ? 1.f / g.dB : 0.f, mt, tig, gid < nhv);
            if (LSE && mt == 0 && gid == 0)
                store_lse<MQ>(p, ub, kvh, hg, nhv, tig, g.mA + ptx::lg2(g.dA), g.mB + ptx::lg2(g.dB));
        }
    }
}

/* ------------------------------------------------------------------------------------ */
/* Host side                                                                            */
/* ------------------------------------------------------------------------------------ */

namespace {

thread_local int g_last_status = PGQA_OK;

int set_status(int s) {
    g_last_status = s;
    return s;
}

int env_int(const char* name, int dflt) {
    const char* v = getenv(name);
    if (v == nullptr || *v == 0) return dflt;
    return atoi(v);
}

/* Sweep knobs (unset in normal use, read once): PGQA_WARPS, PGQA_STAGES, PGQA_MIN_CHUNKS,
 * PGQA_GRID, PGQA_NO_PDL (plain launch instead of a programmatic dependent launch),
 * PGQA_NG (1: one row group per unit even where two would share the K/V tiles),
 * PGQA_SPEC (chunks per warp prefetched into L2 before griddepcontrol.wait; 0: none). */
struct Knobs {
    int warps, stages, min_chunks, grid, no_pdl, ng, spec;
};
const Knobs& knobs() {
    static const Knobs k = {env_int("PGQA_WARPS", 0),      env_int("PGQA_STAGES", 0),
                            env_int("PGQA_MIN_CHUNKS", 0), env_int("PGQA_GRID", 0),
                            env_int("PGQA_NO_PDL", 0),     env_int("PGQA_NG", 0),
                            env_int("PGQA_SPEC", -1)};
    return k;
}

// chunks per warp prefetched into L2 before griddepcontrol.wait (bf16 / e4m3 pools).
// Measured on B200 with the partition kept across the wait: bf16 6 against 4, c2 44.95 ->
// 44.0 us back to back and 53.25 -> 52.3 us isolated, c3 180.1 -> 178.2 us, c4 200.1 ->
// 199.2 us (8: no better, c4 worse); e4m3 4, 6 and 8 within 0.1 us on c2.
constexpr int kDefaultSpecChunks = 6;
constexpr int kDefaultSpecChunksKv8 = 4;
// The pass before griddepcontrol.wait runs when a warp streams at least this many chunks
// on average.  It hides behind a previous decode grid's tail; a call with nothing ahead
// of it pays the pass's two round trips, less what the kept partition saves after the
// wait (c1, isolated behind another kernel: +0.3 to +1.0 us; back to back: -1.4 us).  The
// host checks the table's capacity (the pass is then left out entirely); the kernel
// checks the real lengths before it reads the table and prefetches.
constexpr int64_t kSpecMinChunksPerWarp = 1;

int64_t spec_min_total_for(const pgqa_plan& plan) {
    return kSpecMinChunksPerWarp * plan.grid_ctas * plan.warps_per_cta;
}

int spec_chunks_for(int64_t B, const pgqa_plan& plan, int64_t cap_tokens, bool kv8) {
    if (knobs().spec >= 0) return knobs().spec;
    const int64_t chunks = B * plan.units_per_seq * ((cap_tokens + kChunkTokens - 1) / kChunkTokens);
    if (chunks < spec_min_total_for(plan)) return 0;
    return kv8 ? kDefaultSpecChunksKv8 : kDefaultSpecChunks;
}

// The tensor-core (tcgen05) variant, for KV heads with at most kTcMaxRows query rows.
// Measured on B200 against the mma.sync kernel, it is faster for bf16 pools with more than
// 16 query rows per KV head (several query tokens) over long sequences -- four tokens:
// 0.86x the time on c2, 0.76x on c4, 0.62x on c5 -- and slower for short sequences (1.27x
// on c3, where every unit costs it a fixed epilogue and a partial tile), for one query
// token (1.21x on c2) and for e4m3 pools (1.74x on c2: the V tiles must be converted to
// f16 on the way).  The table capacity stands in for the lengths, which only the device
// reads.  PGQA_TC (read per call) overrides: 1 runs the variant wherever it applies, 0
// never.
constexpr int kTcMinChunks = 8;           // at least one 128-token tile per active CTA
constexpr int64_t kTcMinCapacity = 8192;  // tokens of table capacity for the default choice

bool use_tc(int64_t rows, int64_t Sq, bool kv8, int64_t cap_tokens, size_t smem, int smem_optin) {
    if (rows > kTcMaxRows || smem > (size_t)smem_optin) return false;
    const int forced = env_int("PGQA_TC", -1);
    if (forced >= 0) return forced == 1;
    return !kv8 && Sq > 1 && rows > 16 && cap_tokens >= kTcMinCapacity;
}

constexpr int kDefaultWarps = 8;
constexpr int kDefaultStages = 2;
constexpr int kDefaultStagesKv8 = 4;  // 4 KB stages: the same bytes in flight as 2 x 8 KB
constexpr int kDefaultMinChunks = 2;
constexpr int kB200Sms = 148;
constexpr int kB200SmemOptin = 232448;

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

int smem_bytes_for(int warps, int stages, int64_t B, bool kv8, int ng) {
    size_t s = 1024;  // alignment slack for the 1024-byte aligned ring
    s += (size_t)warps * stages * (kv8 ? kStageBytesKv8 : kStageBytes);
    s += (size_t)warps * stages * 8;
    s += (size_t)(32 + 4 * warps * ng) * 4;      // warp sums + parked keys
    s += align_up((size_t)(B + 1) * 4, 16) + 16;  // prefix table (+ alignment of what follows)
    if (kv8 || ng > 1) s += (size_t)warps * ng * sizeof(Stash);  // early stash slots
    return (int)s;
}

/* Row groups per unit: 2 where a KV head has more than one group of 8 query rows and
 * the (warps, stages) pair has a two-group instantiation. */
bool ng2_compiled(int w, int s, bool kv8) { return w == 8 && s == (kv8 ? 4 : 2); }

/* Instantiated (warps, stages) pairs.  A warp's two parked states reuse its own ring,
 * so every pair must give a ring of at least 2 * sizeof(Stash) per warp. */
bool variant_compiled(int w, int s, bool kv8) {
    if (kv8) return (w == 8 && (s == 3 || s == 4 || s == 6)) || (w == 12 && s == 3);
    return (w == 4 && (s >= 3 && s <= 6)) || (w == 8 && (s == 2 || s == 3));
}

int validate_shape(int64_t B, int64_t Hq, int64_t Hkv, int64_t D, int64_t P) {
    if (B <= 0 || Hq <= 0 || Hkv <= 0 || D <= 0 || P <= 0) return PGQA_ERR_BAD_SHAPE;
    if (Hq % Hkv != 0) return PGQA_ERR_BAD_SHAPE;
    if (D != kHeadDim) return PGQA_ERR_UNSUPPORTED;
    if (P % kChunkTokens != 0) return PGQA_ERR_UNSUPPORTED;
    if (B > (1 << 24) || Hq > 4096) return PGQA_ERR_UNSUPPORTED;
    return PGQA_OK;
}

/* Workspace layout: [error word | record lse | record o | arrival counters].  The record
 * regions depend only on the grid (sized for the largest row-group count per unit), so
 * the counters start at the same offset for every shape: a workspace reused across
 * shapes never reads old records as counters. */
constexpr int kMaxGroupsPerUnit = 2;
size_t record_lse_bytes(int grid) {
    return align_up((size_t)2 * grid * kMaxGroupsPerUnit * 8 * 8 * 4, 256);
}

size_t records_bytes(int grid) {
    return record_lse_bytes(grid) +
           align_up((size_t)2 * grid * kMaxGroupsPerUnit * 8 * kHeadDim * 4, 256);
}

int64_t workspace_bytes_for(int64_t B, int64_t U, int ng, int grid) {
    size_t s = 256;                                   // error word (+ pad)
    s += records_bytes(grid);                         // record lse + record o
    s += align_up((size_t)B * U * ng * 8 * 4, 256);   // arrival counters per row group, M tile
    return (int64_t)s;
}

int make_plan_impl(int64_t B, int64_t Sq, int64_t Hq, int64_t Hkv, int64_t D, int64_t P, int sms,
                   int smem_optin, pgqa_plan* plan, bool kv8 = false) {
    memset(plan, 0, sizeof(*plan));
    int st = validate_shape(B, Hq, Hkv, D, P);
    if (st == PGQA_OK && (Sq <= 0 || Sq > 4096)) st = Sq <= 0 ? PGQA_ERR_BAD_SHAPE : PGQA_ERR_UNSUPPORTED;
    plan->status = st;
    if (st != PGQA_OK) return st;
    if (sms <= 0) sms = kB200Sms;
    if (smem_optin <= 0) smem_optin = kB200SmemOptin;
    const int64_t g = Hq / Hkv;
    // groups of 8 query rows per KV head; row r = (head r / Sq, token r % Sq)
    const int64_t n_hg = ceil_div64(g * Sq, kHeadsPerGroup);
    const Knobs& kn = knobs();
    int w = kn.warps > 0 ? kn.warps : kDefaultWarps;
    int s = kn.stages > 0 ? kn.stages : (kv8 ? kDefaultStagesKv8 : (w == 4 ? 6 : kDefaultStages));
    if (!variant_compiled(w, s, kv8)) {
        // a sweep knob that names no instantiation of this page format: use the defaults
        w = kDefaultWarps;
        s = kv8 ? kDefaultStagesKv8 : kDefaultStages;
    }
    // Two row groups per unit when they exist and that instantiation fits as it is.
    int ng = (n_hg >= 2 && kn.ng != 1 && ng2_compiled(w, s, kv8) &&
              smem_bytes_for(w, s, B, kv8, 2) <= smem_optin) ? 2 : 1;
    // Deepest ring that fits next to the per-sequence prefix table.
    while (smem_bytes_for(w, s, B, kv8, ng) > smem_optin && variant_compiled(w, s - 1, kv8)) --s;
    if (smem_bytes_for(w, s, B, kv8, ng) > smem_optin) {
        plan->status = PGQA_ERR_UNSUPPORTED;  // batch too large for the in-CTA prefix table
        return plan->status;
    }
    plan->warps_per_cta = w;
    plan->stages = s;
    plan->grid_ctas = kn.grid > 0 ? kn.grid : sms;
    plan->min_chunks_per_warp = kn.min_chunks > 0 ? kn.min_chunks : kDefaultMinChunks;
    const int64_t n_w = ceil_div64(n_hg, ng);
    plan->head_groups = (int32_t)n_hg;
    plan->groups_per_unit = ng;
    plan->units_per_seq = (int32_t)(Hkv * n_w);
    plan->smem_bytes = smem_bytes_for(w, s, B, kv8, ng);
    plan->workspace_bytes = workspace_bytes_for(B, Hkv * n_w, ng, plan->grid_ctas);
    plan->status = PGQA_OK;
    return PGQA_OK;
}

/* ---- device properties, cached per device ---- */
struct DevInfo {
    bool init = false;
    int status = PGQA_OK;
    int sms = 0, smem_optin = 0;
};
constexpr int kMaxDevices = 64;
DevInfo g_dev[kMaxDevices];
std::mutex g_dev_mu;

int device_info(int dev, DevInfo* out) {
    if (dev < 0 || dev >= kMaxDevices) return PGQA_ERR_NO_DEVICE;
    std::lock_guard<std::mutex> lk(g_dev_mu);
    DevInfo& d = g_dev[dev];
    if (!d.init) {
        cudaDeviceProp prop;
        if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) {
            cudaGetLastError();
            d.status = PGQA_ERR_NO_DEVICE;
        } else if (prop.major != 10) {
            d.status = PGQA_ERR_NO_DEVICE;  // built for sm_100a only
        } else {
            d.sms = prop.multiProcessorCount;
            d.smem_optin = (int)prop.sharedMemPerBlockOptin;
            d.status = PGQA_OK;
        }
        d.init = true;
    }
    *out = d;
    return d.status;
}

/* ---- cuTensorMapEncodeTiled through the runtime's driver entry point ---- */
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, []() {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess) {
            fn = reinterpret_cast<EncodeTiledFn>(ptr);
        } else {
            cudaGetLastError();
        }
    });
    return fn;
}

/* Tensor map over one pool viewed as (d: 128, kv: Hkv, token: num_pages*P), box
 * (64, 1, 16), 128-byte swizzle.  Out-of-range boxes read zeros (no fault). */
int encode_pool_map(CUtensorMap* map, const void* base, int64_t Hkv, int64_t tokens,
                    bool kv8 = false) {
    EncodeTiledFn fn = encode_fn();
    if (fn == nullptr) return PGQA_ERR_CUDA;
    // FP8 pools: (d: 128 bytes, kv, token), box (128, 1, 16) -- one 2 KB box per chunk
    const cuuint64_t row = kv8 ? kHeadDim : kHeadDim * 2;
    cuuint64_t dims[3] = {(cuuint64_t)kHeadDim, (cuuint64_t)Hkv, (cuuint64_t)tokens};
    cuuint64_t strides[2] = {row, (cuuint64_t)Hkv * row};
    cuuint32_t box[3] = {kv8 ? 128u : 64u, 1, (cuuint32_t)kChunkTokens};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(map, kv8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3,
                    const_cast<void*>(base), dims,
                    strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    // promote to the token row's own size: a 256-byte promotion of a 128-byte
                    // e4m3 row also fetches the neighbouring KV head's row, read much later
                    kv8 ? CU_TENSOR_MAP_L2_PROMOTION_L2_128B : CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? PGQA_OK : PGQA_ERR_CUDA;
}

/* ---- per-device library workspace for run_kernel ---- */
struct LibWorkspace {
    void* ptr = nullptr;
    size_t bytes = 0;
};
LibWorkspace g_ws[kMaxDevices];
std::mutex g_ws_mu;

int lib_workspace(int dev, size_t need, void** out) {
    std::lock_guard<std::mutex> lk(g_ws_mu);
    LibWorkspace& w = g_ws[dev];
    if (w.ptr == nullptr || w.bytes < need) {
        // Test hook: PGQA_DEBUG_FAIL_WORKSPACE_ALLOC=1 makes this allocation fail (the
        // environment is read only here, when an allocation is due).
        if (env_int("PGQA_DEBUG_FAIL_WORKSPACE_ALLOC", 0) != 0) return PGQA_ERR_WORKSPACE;
        if (w.ptr != nullptr) {
            cudaDeviceSynchronize();
            cudaFree(w.ptr);
            w.ptr = nullptr;
            w.bytes = 0;
        }
        size_t sz = need < ((size_t)4 << 20) ? ((size_t)4 << 20) : need;
        if (cudaMalloc(&w.ptr, sz) != cudaSuccess) {
            cudaGetLastError();
            w.ptr = nullptr;
            return PGQA_ERR_WORKSPACE;
        }
        if (cudaMemset(w.ptr, 0, sz) != cudaSuccess) {
            cudaGetLastError();
            return PGQA_ERR_CUDA;
        }
        w.bytes = sz;
    }
    *out = w.ptr;
    return PGQA_OK;
}

template <int W, int S, bool MQ, bool KV8, int NG, bool LSE = false>
int launch_variant(const CUtensorMap& km, const CUtensorMap& vm, const DecodeParams& p, int grid,
                   int smem, cudaStream_t stream) {
    auto kern = pgqa_decode_kernel<W, S, MQ, KV8, NG, LSE>;
    static int configured_smem[kMaxDevices] = {0};  // one table per instantiation
    int dev = 0;
    cudaGetDevice(&dev);
    if (configured_smem[dev] < smem) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
            cudaSuccess) {
            cudaGetLastError();
            return PGQA_ERR_CUDA;
        }
        configured_smem[dev] = smem;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(W * 32);
    cfg.dynamicSmemBytes = (size_t)smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = knobs().no_pdl ? 0 : 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, km, vm, p);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return PGQA_ERR_CUDA;
    }
    return PGQA_OK;
}

template <bool MQ, bool KV8>
int launch_t(const pgqa_plan& plan, const CUtensorMap& km, const CUtensorMap& vm,
             const DecodeParams& p, cudaStream_t stream) {
    const int w = plan.warps_per_cta, s = plan.stages;
    const int g = plan.grid_ctas, sm = plan.smem_bytes;
    if (p.lse_out != nullptr) {
        // the log-sum-exp output is compiled for the default rings only (8 warps; bf16
        // 2 stages, e4m3 4) so that no other instantiation carries its code
        if (w != 8 || s != (KV8 ? 4 : 2)) return PGQA_ERR_UNSUPPORTED;
        if (plan.groups_per_unit == 2)
            return launch_variant<8, KV8 ? 4 : 2, MQ, KV8, 2, true>(km, vm, p, g, sm, stream);
        return launch_variant<8, KV8 ? 4 : 2, MQ, KV8, 1, true>(km, vm, p, g, sm, stream);
    }
    if (plan.groups_per_unit == 2) {
        if (KV8 && w == 8 && s == 4) return launch_variant<8, 4, MQ, true, 2>(km, vm, p, g, sm, stream);
        if (!KV8 && w == 8 && s == 2) return launch_variant<8, 2, MQ, false, 2>(km, vm, p, g, sm, stream);
        return PGQA_ERR_UNSUPPORTED;
    }
    if (KV8) {
        if (w == 12 && s == 3) return launch_variant<12, 3, MQ, true, 1>(km, vm, p, g, sm, stream);
        if (w == 8 && s == 4) return launch_variant<8, 4, MQ, true, 1>(km, vm, p, g, sm, stream);
        if (w == 8 && s == 3) return launch_variant<8, 3, MQ, true, 1>(km, vm, p, g, sm, stream);
        if (w == 8 && s == 6) return launch_variant<8, 6, MQ, true, 1>(km, vm, p, g, sm, stream);
        return PGQA_ERR_UNSUPPORTED;
    }
    if (w == 4 && s == 6) return launch_variant<4, 6, MQ, false, 1>(km, vm, p, g, sm, stream);
    if (w == 4 && s == 5) return launch_variant<4, 5, MQ, false, 1>(km, vm, p, g, sm, stream);
    if (w == 4 && s == 4) return launch_variant<4, 4, MQ, false, 1>(km, vm, p, g, sm, stream);
    if (w == 4 && s == 3) return launch_variant<4, 3, MQ, false, 1>(km, vm, p, g, sm, stream);
    if (w == 8 && s == 3) return launch_variant<8, 3, MQ, false, 1>(km, vm, p, g, sm, stream);
    if (w == 8 && s == 2) return launch_variant<8, 2, MQ, false, 1>(km, vm, p, g, sm, stream);
    return PGQA_ERR_UNSUPPORTED;
}

/* One query token (causal or not: an end-aligned mask hides nothing) takes the
 * single-token instantiation. */
int launch(const pgqa_plan& plan, const CUtensorMap& km, const CUtensorMap& vm,
           const DecodeParams& p, bool kv8, cudaStream_t stream) {
    if (kv8)
        return p.Sq > 1 ? launch_t<true, true>(plan, km, vm, p, stream)
                        : launch_t<false, true>(plan, km, vm, p, stream);
    return p.Sq > 1 ? launch_t<true, false>(plan, km, vm, p, stream)
                    : launch_t<false, false>(plan, km, vm, p, stream);
}

int decode_impl(const void* q, const void* k, const void* v, void* out, const int32_t* seq_lens,
                const int32_t* bt, int64_t B, int64_t Sq, int64_t Hq, int64_t Hkv, int64_t D,
                int64_t P, int64_t num_pages, int64_t bt_stride, int64_t max_seqlen,
                int64_t causal, float scale, void* workspace, size_t ws_bytes,
                cudaStream_t stream, const void* k_new = nullptr, const void* v_new = nullptr,
                int64_t len_add = 0, bool kv8 = false, const float* k_scale = nullptr,
                const float* v_scale = nullptr, float* lse_out = nullptr) {
    if (!q || !k || !v || !out || !seq_lens || !bt) return PGQA_ERR_NULL_POINTER;
    if (len_add < 0 || len_add > 4096) return len_add < 0 ? PGQA_ERR_BAD_SHAPE : PGQA_ERR_UNSUPPORTED;
    if (len_add > 0 && (!k_new || !v_new)) return PGQA_ERR_NULL_POINTER;
    if ((reinterpret_cast<uintptr_t>(k_new) & 15) || (reinterpret_cast<uintptr_t>(v_new) & 15) ||
        (reinterpret_cast<uintptr_t>(k_scale) & 3) || (reinterpret_cast<uintptr_t>(v_scale) & 3))
        return PGQA_ERR_MISALIGNED;
    int st = validate_shape(B, Hq, Hkv, D, P);
    if (st != PGQA_OK) return st;
    if (num_pages <= 0 || bt_stride <= 0) return PGQA_ERR_BAD_SHAPE;
    if (num_pages * P >= ((int64_t)1 << 31)) return PGQA_ERR_UNSUPPORTED;
    const int64_t cap = bt_stride * P;
    if (max_seqlen < 0 || max_seqlen > cap) return PGQA_ERR_BAD_SHAPE;
    if (!(scale > 0.f) || !isfinite(scale)) return PGQA_ERR_BAD_SHAPE;
    if (causal != 0 && causal != 1) return PGQA_ERR_BAD_SHAPE;
    if ((reinterpret_cast<uintptr_t>(k) & 15) || (reinterpret_cast<uintptr_t>(v) & 15) ||
        (reinterpret_cast<uintptr_t>(q) & 15) || (reinterpret_cast<uintptr_t>(out) & 15) ||
        (reinterpret_cast<uintptr_t>(seq_lens) & 3) || (reinterpret_cast<uintptr_t>(bt) & 3))
        return PGQA_ERR_MISALIGNED;

    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        return PGQA_ERR_NO_DEVICE;
    }
    DevInfo di;
    st = device_info(dev, &di);
    if (st != PGQA_OK) return st;
    pgqa_plan plan;
    st = make_plan_impl(B, Sq, Hq, Hkv, D, P, di.sms, di.smem_optin, &plan, kv8);
    if (st != PGQA_OK) return st;

    if (workspace == nullptr) {
        st = lib_workspace(dev, (size_t)plan.workspace_bytes, &workspace);
        if (st != PGQA_OK) return st;
    } else if (ws_bytes < (size_t)plan.workspace_bytes) {
        return PGQA_ERR_WORKSPACE;
    }
    if (reinterpret_cast<uintptr_t>(workspace) & 255) return PGQA_ERR_MISALIGNED;

    CUtensorMap km, vm;
    st = encode_pool_map(&km, k, Hkv, num_pages * P, kv8);
    if (st != PGQA_OK) return st;
    st = encode_pool_map(&vm, v, Hkv, num_pages * P, kv8);
    if (st != PGQA_OK) return st;

    const int64_t g = Hq / Hkv;
    DecodeParams p;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    p.err = reinterpret_cast<int32_t*>(ws);
    size_t off = 256;
    p.rec_lse = reinterpret_cast<float*>(ws + off);
    off += record_lse_bytes(plan.grid_ctas);
    p.rec_o = reinterpret_cast<float*>(ws + off);
    off = 256 + records_bytes(plan.grid_ctas);
    p.counters = reinterpret_cast<int32_t*>(ws + off);
    p.q = static_cast<const __nv_bfloat16*>(q);
    p.out = static_cast<__nv_bfloat16*>(out);
    p.lse_out = lse_out;
    p.seq_lens = seq_lens;
    p.block_table = bt;
    p.B = (int32_t)B;
    p.Hq = (int32_t)Hq;
    p.Hkv = (int32_t)Hkv;
    p.g = (int32_t)g;
    p.n_hg = plan.head_groups;
    p.n_w = plan.units_per_seq / (int32_t)Hkv;
    p.U = plan.units_per_seq;
    p.Sq = (int32_t)Sq;
    p.rows = (int32_t)(g * Sq);
    p.causal = (int32_t)causal;
    p.len_add = (int32_t)len_add;
    p.k_scale = k_scale;
    p.v_scale = v_scale;
    p.page_size = (int32_t)P;
    p.page_shift = -1;
    for (int sh = 0; sh < 31; ++sh)
        if (((int64_t)1 << sh) == P) p.page_shift = sh;
    p.bt_stride = (int32_t)bt_stride;
    p.num_pages = (int32_t)num_pages;
    p.cap_tokens = cap;
    p.scale_log2 = scale * 1.4426950408889634f;
    p.min_chunks = plan.min_chunks_per_warp;
    // Test hooks, read per call: PGQA_DEBUG_STUCK_BARRIER=n (n > 0) makes the first stage
    // barrier of warp n-1 in CTA 0 wait for 16 bytes that never arrive (its wait expires
    // -> PGQA_ERR_DEVICE_TIMEOUT);
    // PGQA_WAIT_LIMIT_NS shortens the bound on every wait; PGQA_DEBUG_SPEC_SKEW=n adds n
    // to the lengths the speculative pass sees, as if a predecessor had rewritten them
    // (and runs that pass whatever the size of the call).
    p.debug_stuck = env_int("PGQA_DEBUG_STUCK_BARRIER", 0);
    p.debug_spec_skew = env_int("PGQA_DEBUG_SPEC_SKEW", 0);
    p.spec_chunks = spec_chunks_for(B, plan, cap, kv8);
    // The sweep knob and the test hook run the whole pass whatever the size of the call.
    p.spec_min_total = (knobs().spec >= 0 || p.debug_spec_skew != 0) ? 0 : spec_min_total_for(plan);
    if (p.debug_spec_skew != 0 && p.spec_chunks == 0) p.spec_chunks = kDefaultSpecChunks;
    {
        const char* lim = getenv("PGQA_WAIT_LIMIT_NS");
        p.wait_limit_ns = (lim && *lim) ? strtoull(lim, nullptr, 10) : kWaitLimitNs;
        if (p.wait_limit_ns == 0 || p.wait_limit_ns > 10 * kWaitLimitNs) p.wait_limit_ns = kWaitLimitNs;
    }
    if (len_add > 0) {
        // Append first; the decode launches as its programmatic dependent and its
        // griddepcontrol.wait orders every read of the pool after the append's writes.
        AppendArgs a;
        a.k_new = static_cast<const uint4*>(k_new);
        a.v_new = static_cast<const uint4*>(v_new);
        a.k_cache = static_cast<uint4*>(const_cast<void*>(k));
        a.v_cache = static_cast<uint4*>(const_cast<void*>(v));
        a.seq_lens = seq_lens;
        a.block_table = bt;
        a.err = p.err;
        a.B = (int32_t)B;
        a.S_new = (int32_t)len_add;
        a.Hkv = (int32_t)Hkv;
        a.P = (int32_t)P;
        a.bt_stride = (int32_t)bt_stride;
        a.num_pages = (int32_t)num_pages;
        a.cap_tokens = cap;
        a.row_pieces_log2 = kv8 ? 3 : 4;
        if (launch_append(a, di.sms, stream) != 0) return PGQA_ERR_CUDA;
    }
    const size_t tc_smem = tc_smem_bytes(kv8, (int)(g * Sq), B);
    if (use_tc(g * Sq, Sq, kv8, cap, tc_smem, di.smem_optin)) {
        TcParams t;
        t.q = p.q;
        t.out = p.out;
        t.lse_out = p.lse_out;
        t.seq_lens = p.seq_lens;
        t.block_table = p.block_table;
        t.rec_o = p.rec_o;
        t.rec_lse = p.rec_lse;
        t.counters = p.counters;
        t.err = p.err;
        t.B = p.B;
        t.Hq = p.Hq;
        t.Hkv = p.Hkv;
        t.g = p.g;
        t.Sq = p.Sq;
        t.rows = p.rows;
        t.causal = p.causal;
        t.len_add = p.len_add;
        t.k_scale = p.k_scale;
        t.v_scale = p.v_scale;
        t.page_size = p.page_size;
        t.page_shift = p.page_shift;
        t.bt_stride = p.bt_stride;
        t.num_pages = p.num_pages;
        t.cap_tokens = p.cap_tokens;
        t.scale_log2 = p.scale_log2;
        t.min_chunks = knobs().min_chunks > 0 ? knobs().min_chunks : kTcMinChunks;
        t.debug_stuck = p.debug_stuck;
        t.wait_limit_ns = p.wait_limit_ns;
        if (launch_tc(km, vm, t, kv8, plan.grid_ctas, tc_smem, knobs().no_pdl == 0, stream) !=
            cudaSuccess) {
            cudaGetLastError();
            return PGQA_ERR_CUDA;
        }
        return PGQA_OK;
    }
    return launch(plan, km, vm, p, kv8, stream);
}

}  // namespace
}  // namespace pgqa

/* ------------------------------------------------------------------------------------ */
/* C ABI                                                                                */
/* ------------------------------------------------------------------------------------ */

using namespace pgqa;

extern "C" void run_kernel(const void* q, const void* k_cache_paged, const void* v_cache_paged,
                           void* output, const int32_t* cache_seqlens,
                           const int32_t* block_table, int64_t batch_size, int64_t seqlen_k,
                           int64_t seqlen_q, int64_t num_heads, int64_t num_heads_k,
                           int64_t headdim, int64_t page_block_size, int64_t num_blocks,
                           int64_t causal) {
    if (batch_size <= 0 || num_blocks <= 0 || num_blocks % batch_size != 0 || seqlen_k < 0 ||
        page_block_size <= 0) {
        set_status(PGQA_ERR_BAD_SHAPE);
        return;
    }
    // seqlen_q query tokens per sequence; causal aligns the mask to the end of the
    // cache (token i sees keys [0, L - seqlen_q + i]).  With one token it hides nothing.
    if (seqlen_q <= 0 || (causal != 0 && causal != 1)) {
        set_status(seqlen_q <= 0 ? PGQA_ERR_BAD_SHAPE : PGQA_ERR_UNSUPPORTED);
        return;
    }
    const int64_t stride = num_blocks / batch_size;
    if (seqlen_k > stride * page_block_size) {
        set_status(PGQA_ERR_BAD_SHAPE);
        return;
    }
    const float scale = 1.0f / sqrtf((float)headdim);
    set_status(decode_impl(q, k_cache_paged, v_cache_paged, output, cache_seqlens, block_table,
                           batch_size, seqlen_q, num_heads, num_heads_k, headdim, page_block_size,
                           num_blocks, stride, seqlen_k, causal, scale, nullptr, 0,
                           (cudaStream_t)0));
}

extern "C" int pgqa_decode_v1(const void* q, const void* k_cache, const void* v_cache, void* out,
                              const int32_t* seq_lens, const int32_t* block_table,
                              int64_t batch_size, int64_t num_heads, int64_t num_heads_k,
                              int64_t headdim, int64_t page_size, int64_t num_pages,
                              int64_t bt_stride, int64_t max_seqlen, float scale,
                              void* workspace, size_t workspace_bytes, void* stream) {
    return set_status(decode_impl(q, k_cache, v_cache, out, seq_lens, block_table, batch_size, 1,
                                  num_heads, num_heads_k, headdim, page_size, num_pages, bt_stride,
                                  max_seqlen, 0, scale, workspace, workspace_bytes,
                                  static_cast<cudaStream_t>(stream)));
}

extern "C" int pgqa_decode_v2(const void* q, const void* k_cache, const void* v_cache, void* out,
                              const int32_t* seq_lens, const int32_t* block_table,
                              int64_t batch_size, int64_t seqlen_q, int64_t num_heads,
                              int64_t num_heads_k, int64_t headdim, int64_t page_size,
                              int64_t num_pages, int64_t bt_stride, int64_t max_seqlen,
                              int64_t causal, float scale, void* workspace,
                              size_t workspace_bytes, void* stream) {
    return set_status(decode_impl(q, k_cache, v_cache, out, seq_lens, block_table, batch_size,
                                  seqlen_q, num_heads, num_heads_k, headdim, page_size, num_pages,
                                  bt_stride, max_seqlen, causal, scale, workspace,
                                  workspace_bytes, static_cast<cudaStream_t>(stream)));
}

extern "C" int pgqa_decode_kvcache(const void* q, void* k_cache, void* v_cache,
                                   const void* k_new, const void* v_new, void* out,
                                   const int32_t* seq_lens, const int32_t* block_table,
                                   int64_t batch_size, int64_t seqlen_q, int64_t seqlen_new,
                                   int64_t num_heads, int64_t num_heads_k, int64_t headdim,
                                   int64_t page_size, int64_t num_pages, int64_t bt_stride,
                                   int64_t max_seqlen, int64_t causal, float scale,
                                   void* workspace, size_t workspace_bytes, void* stream) {
    return set_status(decode_impl(q, k_cache, v_cache, out, seq_lens, block_table, batch_size,
                                  seqlen_q, num_heads, num_heads_k, headdim, page_size, num_pages,
                                  bt_stride, max_seqlen, causal, scale, workspace,
                                  workspace_bytes, static_cast<cudaStream_t>(stream), k_new,
                                  v_new, seqlen_new));
}

namespace {
int append_entry(const void* k_new, const void* v_new, void* k_cache, void* v_cache,
                 const int32_t* seq_lens, const int32_t* block_table, int64_t batch_size,
                 int64_t seqlen_new, int64_t num_heads_k, int64_t headdim, int64_t page_size,
                 int64_t num_pages, int64_t bt_stride, void* workspace, void* stream, bool kv8) {
    if (!k_new || !v_new || !k_cache || !v_cache || !seq_lens || !block_table)
        return PGQA_ERR_NULL_POINTER;
    if (batch_size <= 0 || seqlen_new < 0 || num_heads_k <= 0 || page_size <= 0 ||
        num_pages <= 0 || bt_stride <= 0 || batch_size > INT32_MAX || seqlen_new > INT32_MAX ||
        num_heads_k > INT32_MAX || page_size > INT32_MAX || num_pages > INT32_MAX ||
        bt_stride > INT32_MAX)
        return PGQA_ERR_BAD_SHAPE;
    if (headdim != kHeadDim) return PGQA_ERR_UNSUPPORTED;
    if ((reinterpret_cast<uintptr_t>(k_new) & 15) || (reinterpret_cast<uintptr_t>(v_new) & 15) ||
        (reinterpret_cast<uintptr_t>(k_cache) & 15) || (reinterpret_cast<uintptr_t>(v_cache) & 15) ||
        (reinterpret_cast<uintptr_t>(seq_lens) & 3) || (reinterpret_cast<uintptr_t>(block_table) & 3))
        return PGQA_ERR_MISALIGNED;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        return PGQA_ERR_NO_DEVICE;
    }
    DevInfo di;
    int st = device_info(dev, &di);
    if (st != PGQA_OK) return st;
    if (workspace == nullptr) {
        st = lib_workspace(dev, 256, &workspace);
        if (st != PGQA_OK) return st;
    }
    AppendArgs a;
    a.k_new = static_cast<const uint4*>(k_new);
    a.v_new = static_cast<const uint4*>(v_new);
    a.k_cache = static_cast<uint4*>(k_cache);
    a.v_cache = static_cast<uint4*>(v_cache);
    a.seq_lens = seq_lens;
    a.block_table = block_table;
    a.err = static_cast<int32_t*>(workspace);
    a.B = (int32_t)batch_size;
    a.S_new = (int32_t)seqlen_new;
    a.Hkv = (int32_t)num_heads_k;
    a.P = (int32_t)page_size;
    a.bt_stride = (int32_t)bt_stride;
    a.num_pages = (int32_t)num_pages;
    a.cap_tokens = bt_stride * page_size;
    a.row_pieces_log2 = kv8 ? 3 : 4;
    if (launch_append(a, di.sms, static_cast<cudaStream_t>(stream)) != 0) return PGQA_ERR_CUDA;
    return PGQA_OK;
}
}  // namespace

extern "C" int pgqa_append_kv(const void* k_new, const void* v_new, void* k_cache,
                              void* v_cache, const int32_t* seq_lens,
                              const int32_t* block_table, int64_t batch_size, int64_t seqlen_new,
                              int64_t num_heads_k, int64_t headdim, int64_t page_size,
                              int64_t num_pages, int64_t bt_stride, void* workspace,
                              void* stream) {
    return set_status(append_entry(k_new, v_new, k_cache, v_cache, seq_lens, block_table,
                                   batch_size, seqlen_new, num_heads_k, headdim, page_size,
                                   num_pages, bt_stride, workspace, stream, false));
}

extern "C" int pgqa_append_kv_fp8(const void* k_new, const void* v_new, void* k_cache,
                                  void* v_cache, const int32_t* seq_lens,
                                  const int32_t* block_table, int64_t batch_size,
                                  int64_t seqlen_new, int64_t num_heads_k, int64_t headdim,
                                  int64_t page_size, int64_t num_pages, int64_t bt_stride,
                                  void* workspace, void* stream) {
    return set_status(append_entry(k_new, v_new, k_cache, v_cache, seq_lens, block_table,
                                   batch_size, seqlen_new, num_heads_k, headdim, page_size,
                                   num_pages, bt_stride, workspace, stream, true));
}

extern "C" int pgqa_decode_fp8(const void* q, void* k_cache, void* v_cache, const void* k_new,
                               const void* v_new, void* out, const int32_t* seq_lens,
                               const int32_t* block_table, int64_t batch_size, int64_t seqlen_q,
                               int64_t seqlen_new, int64_t num_heads, int64_t num_heads_k,
                               int64_t headdim, int64_t page_size, int64_t num_pages,
                               int64_t bt_stride, int64_t max_seqlen, int64_t causal, float scale,
                               const float* k_scale, const float* v_scale, void* workspace,
                               size_t workspace_bytes, void* stream) {
    return set_status(decode_impl(q, k_cache, v_cache, out, seq_lens, block_table, batch_size,
                                  seqlen_q, num_heads, num_heads_k, headdim, page_size, num_pages,
                                  bt_stride, max_seqlen, causal, scale, workspace,
                                  workspace_bytes, static_cast<cudaStream_t>(stream), k_new,
                                  v_new, seqlen_new, true, k_scale, v_scale));
}

extern "C" int pgqa_decode_ex(const pgqa_decode_args* a, void* stream) {
    if (a == nullptr) return set_status(PGQA_ERR_NULL_POINTER);
    if (a->struct_size != sizeof(pgqa_decode_args)) return set_status(PGQA_ERR_BAD_SHAPE);
    if (a->kv_format != 0 && a->kv_format != 1) return set_status(PGQA_ERR_UNSUPPORTED);
    if (a->kv_format == 0 && (a->k_scale != nullptr || a->v_scale != nullptr))
        return set_status(PGQA_ERR_BAD_SHAPE);  // scales describe e4m3 pools only
    if (reinterpret_cast<uintptr_t>(a->softmax_lse) & 3) return set_status(PGQA_ERR_MISALIGNED);
    return set_status(decode_impl(a->q, a->k_cache, a->v_cache, a->out, a->seq_lens,
                                  a->block_table, a->batch_size, a->seqlen_q, a->num_heads,
                                  a->num_heads_k, a->headdim, a->page_size, a->num_pages,
                                  a->bt_stride, a->max_seqlen, a->causal, a->scale, a->workspace,
                                  a->workspace_bytes, static_cast<cudaStream_t>(stream),
                                  a->k_new, a->v_new, a->seqlen_new, a->kv_format == 1,
                                  a->k_scale, a->v_scale, a->softmax_lse));
}

static size_t workspace_size_impl(int64_t batch_size, int64_t seqlen_q, int64_t num_heads,
                                  int64_t num_heads_k, int64_t headdim, int64_t page_size) {
    int sms = 0, optin = 0;
    int dev = 0;
    DevInfo di;
    if (cudaGetDevice(&dev) == cudaSuccess && device_info(dev, &di) == PGQA_OK) {
        sms = di.sms;
        optin = di.smem_optin;
    } else {
        cudaGetLastError();
    }
    pgqa_plan plan;
    // the reason for a 0 (bad or unsupported shape) is left for pgqa_last_status()
    if (set_status(make_plan_impl(batch_size, seqlen_q, num_heads, num_heads_k, headdim,
                                  page_size, sms, optin, &plan)) != PGQA_OK)
        return 0;
    return (size_t)plan.workspace_bytes;
}

extern "C" size_t pgqa_workspace_size(int64_t batch_size, int64_t num_heads, int64_t num_heads_k,
                                      int64_t headdim, int64_t page_size) {
    return workspace_size_impl(batch_size, 1, num_heads, num_heads_k, headdim, page_size);
}

extern "C" size_t pgqa_workspace_size_v2(int64_t batch_size, int64_t seqlen_q, int64_t num_heads,
                                         int64_t num_heads_k, int64_t headdim, int64_t page_size) {
    return workspace_size_impl(batch_size, seqlen_q, num_heads, num_heads_k, headdim, page_size);
}

extern "C" int pgqa_workspace_init(void* workspace, size_t workspace_bytes, void* stream) {
    if (workspace == nullptr) return set_status(PGQA_ERR_NULL_POINTER);
    if (cudaMemsetAsync(workspace, 0, workspace_bytes, static_cast<cudaStream_t>(stream)) !=
        cudaSuccess) {
        cudaGetLastError();
        return set_status(PGQA_ERR_CUDA);
    }
    return set_status(PGQA_OK);
}

extern "C" int pgqa_last_status(void) { return g_last_status; }

extern "C" const char* pgqa_status_string(int status) {
    switch (status) {
        case PGQA_OK: return "ok";
        case PGQA_ERR_NULL_POINTER: return "null pointer argument";
        case PGQA_ERR_BAD_SHAPE: return "invalid shape argument";
        case PGQA_ERR_UNSUPPORTED: return "unsupported configuration";
        case PGQA_ERR_MISALIGNED: return "misaligned pointer";
        case PGQA_ERR_WORKSPACE: return "workspace missing, too small or not allocatable";
        case PGQA_ERR_CUDA: return "CUDA call failed";
        case PGQA_ERR_NO_DEVICE: return "no usable sm_100 device";
        case PGQA_ERR_DEVICE_TIMEOUT: return "device-side wait timed out";
        case PGQA_ERR_DEVICE_BAD_PAGE: return "block_table entry outside [0, num_pages)";
        case PGQA_ERR_DEVICE_BAD_SEQLEN: return "seq_len outside [0, table capacity]";
        case PGQA_ERR_SCRATCH_LIMIT:
            return "shape needs more scratch than the fixed 4 MiB allocation-free buffer";
        default: return "unknown status";
    }
}

namespace {
/* Waits for `s`, reads the 4-byte device error word at `word_ptr`, clears it when it is
 * set, and maps its bits to a status. */
int read_error_word(void* word_ptr, cudaStream_t s) {
    int32_t word = 0;
    if (cudaMemcpyAsync(&word, word_ptr, 4, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess) {
        cudaGetLastError();
        return PGQA_ERR_CUDA;
    }
    if (word != 0) {
        cudaMemsetAsync(word_ptr, 0, 4, s);
        cudaStreamSynchronize(s);
    }
    if (word & kErrTimeout) return PGQA_ERR_DEVICE_TIMEOUT;
    if (word & kErrBadPage) return PGQA_ERR_DEVICE_BAD_PAGE;
    if (word & kErrBadSeqlen) return PGQA_ERR_DEVICE_BAD_SEQLEN;
    return PGQA_OK;
}
}  // namespace

extern "C" int pgqa_check_device_error(void* workspace, void* stream) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        return PGQA_ERR_NO_DEVICE;
    }
    if (workspace == nullptr) {
        std::lock_guard<std::mutex> lk(g_ws_mu);
        if (dev < 0 || dev >= kMaxDevices || g_ws[dev].ptr == nullptr) return PGQA_OK;
        workspace = g_ws[dev].ptr;
    }
    return read_error_word(workspace, static_cast<cudaStream_t>(stream));
}

extern "C" int pgqa_make_plan(int64_t batch_size, int64_t num_heads, int64_t num_heads_k,
                              int64_t headdim, int64_t page_size, int32_t num_sms,
                              int32_t smem_per_block_optin, pgqa_plan* plan) {
    if (plan == nullptr) return PGQA_ERR_NULL_POINTER;
    return make_plan_impl(batch_size, 1, num_heads, num_heads_k, headdim, page_size, num_sms,
                          smem_per_block_optin, plan);
}

extern "C" int64_t pgqa_simulate_partition(const int32_t* seq_lens, int64_t B, int64_t U,
                                           int64_t cap_tokens, const pgqa_plan* plan,
                                           int32_t* ctas_per_unit, int32_t* segments_per_unit) {
    if (!seq_lens || !plan || !ctas_per_unit || !segments_per_unit) return -PGQA_ERR_NULL_POINTER;
    if (B <= 0 || U <= 0 || plan->grid_ctas <= 0 || plan->warps_per_cta <= 0) return -PGQA_ERR_BAD_SHAPE;
    int64_t* pre = static_cast<int64_t*>(malloc(sizeof(int64_t) * (B + 1)));
    if (!pre) return -PGQA_ERR_WORKSPACE;
    pre[0] = 0;
    for (int64_t b = 0; b < B; ++b) pre[b + 1] = pre[b] + seq_chunks(seq_lens[b], cap_tokens);
    for (int64_t u = 0; u < B * U; ++u) ctas_per_unit[u] = segments_per_unit[u] = 0;
    const int64_t T = pre[B] * U;
    if (T == 0) {
        free(pre);
        return 0;
    }
    auto unit_of = [&](int64_t x) -> int64_t {  // flat unit index containing chunk x
        int64_t lo = 0, hi = B;
        while (hi - lo > 1) {
            const int64_t mid = (lo + hi) / 2;
            if (pre[mid] * U <= x) lo = mid; else hi = mid;
        }
        const int64_t n = pre[lo + 1] - pre[lo];
        return lo * U + (x - pre[lo] * U) / n;
    };
    const int64_t W = plan->warps_per_cta;
    bool uniform = true;
    for (int64_t b = 1; b < B; ++b)
        if (pre[b + 1] - pre[b] != pre[1] - pre[0]) uniform = false;
    uniform = uniform && pre[1] > 0;
    const int64_t nct = align_ctas(active_ctas(T, plan->grid_ctas, W, plan->min_chunks_per_warp), B * U, uniform);
    for (int64_t c = 0; c < nct; ++c) {
        const int64_t cs = slice_begin(c, nct, T), ce = slice_begin(c + 1, nct, T);
        for (int64_t u = unit_of(cs); u <= unit_of(ce - 1); ++u) ctas_per_unit[u] += 1;
        const int64_t len = ce - cs;
        const int64_t wa = active_warps(len, W);
        for (int64_t w = 0; w < wa; ++w) {
            const int64_t ws = cs + slice_begin(w, wa, len), we = cs + slice_begin(w + 1, wa, len);
            for (int64_t u = unit_of(ws); u <= unit_of(we - 1); ++u) segments_per_unit[u] += 1;
        }
    }
    free(pre);
    return nct;
}

extern "C" const char* pgqa_version(void) { return "pgqa-b200 0.1 (sm_100a)"; }

/* ------------------------------------------------------------------------------------ */
/* Allocation-free entry point                                                          */
/* ------------------------------------------------------------------------------------ */

/* Scratch for pgqa_decode_noalloc: the same layout pgqa_decode_v1 expects of a caller's
 * workspace (error word, split records, arrival counters), held in a fixed array that
 * every GPU loading this library keeps until the process exits.  On a 148-SM B200 the
 * records take 2.58 MB (sized for two row groups per unit), leaving 50,552 arrival-
 * counter entries of 32 bytes, one per (sequence, unit, row group): B * Hkv at up to 8
 * query heads per KV head, B * Hkv * 2 * ceil(ceil(g/8)/2) beyond. */
constexpr size_t kNoAllocScratchBytes = (size_t)4 << 20;
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

namespace {
struct NoAllocScratch {
    bool init = false;
    int status = PGQA_OK;
    void* ptr = nullptr;  // device address of g_noalloc_scratch on this device
};
NoAllocScratch g_noalloc[pgqa::kMaxDevices];
std::mutex g_noalloc_mu;

/* Host code may not use g_noalloc_scratch itself (that name is a host-side stand-in,
 * not a device address): resolve the device address once per device, with that device
 * current.  *fresh is set on the call that did the look-up. */
int noalloc_scratch(int dev, void** out, bool* fresh) {
    *fresh = false;
    if (dev < 0 || dev >= pgqa::kMaxDevices) return PGQA_ERR_NO_DEVICE;
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    NoAllocScratch& s = g_noalloc[dev];
    if (!s.init) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || p == nullptr) {
            cudaGetLastError();
            s.status = PGQA_ERR_CUDA;
        } else {
            s.ptr = p;
            s.status = PGQA_OK;
            *fresh = true;
        }
        s.init = true;
    }
    *out = s.ptr;
    return s.status;
}
}  // namespace

extern "C" int pgqa_decode_noalloc(const void* q, const void* k_cache, const void* v_cache,
                                   void* out, const int32_t* seq_lens,
                                   const int32_t* block_table, int64_t batch_size,
                                   int64_t num_heads, int64_t num_heads_k, int64_t headdim,
                                   int64_t page_size, int64_t num_pages, int64_t bt_stride,
                                   int64_t max_seqlen, float scale, void* stream) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        return set_status(PGQA_ERR_NO_DEVICE);
    }
    DevInfo di;
    int st = device_info(dev, &di);
    if (st != PGQA_OK) return set_status(st);
    pgqa_plan plan;
    st = make_plan_impl(batch_size, 1, num_heads, num_heads_k, headdim, page_size, di.sms,
                        di.smem_optin, &plan);
    if (st != PGQA_OK) return set_status(st);
    if ((size_t)plan.workspace_bytes > kNoAllocScratchBytes)
        return set_status(PGQA_ERR_SCRATCH_LIMIT);
    void* scratch = nullptr;
    bool fresh = false;
    st = noalloc_scratch(dev, &scratch, &fresh);
    if (st != PGQA_OK) return set_status(st);
    // The array keeps the previous call's contents.  The arrival counters must start at
    // zero for every call (the kernel leaves them zeroed, this is a second guard).  The
    // error word is cleared once, at set-up, and otherwise only by
    // pgqa_noalloc_check_device_error: an error stays readable until the caller reads it.
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    uint8_t* base = static_cast<uint8_t*>(scratch);
    const size_t counters_off = 256 + records_bytes(plan.grid_ctas);
    const size_t counters_len = (size_t)plan.workspace_bytes - counters_off;
    if ((fresh && cudaMemsetAsync(base, 0, 256, s) != cudaSuccess) ||
        cudaMemsetAsync(base + counters_off, 0, counters_len, s) != cudaSuccess) {
        cudaGetLastError();
        return set_status(PGQA_ERR_CUDA);
    }
    return set_status(decode_impl(q, k_cache, v_cache, out, seq_lens, block_table, batch_size, 1,
                                  num_heads, num_heads_k, headdim, page_size, num_pages,
                                  bt_stride, max_seqlen, 0, scale, scratch, kNoAllocScratchBytes,
                                  s));
}


extern "C" int pgqa_noalloc_check_device_error(void* stream) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        return PGQA_ERR_NO_DEVICE;
    }
    if (dev < 0 || dev >= pgqa::kMaxDevices) return PGQA_ERR_NO_DEVICE;
    void* scratch = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_noalloc_mu);
        const NoAllocScratch& sc = g_noalloc[dev];
        if (!sc.init || sc.status != PGQA_OK) return PGQA_OK;  // no call has run here
        scratch = sc.ptr;
    }
    return read_error_word(scratch, static_cast<cudaStream_t>(stream));
}
