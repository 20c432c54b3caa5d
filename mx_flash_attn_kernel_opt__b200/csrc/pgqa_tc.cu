/*
 * pgqa_tc.cu - paged grouped-query-attention decode on the 5th-generation tensor core
 * (tcgen05 MMAs with TMEM accumulators), for the two paths whose mma.sync form is bound
 * by instruction issue rather than by HBM:
 *   - e4m3 KV pages (K goes to the tensor core as stored, QK^T in kind::f8f6f4), and
 *   - several query tokens per sequence (speculative / multi-token decode).
 * It replaces the same reference stages as pgqa_decode.cu -- the split-KV partial kernel
 * (submission_clean.cu:66-300; its MMA sites :182-216), the split combine
 * (submission_clean.cu:307-360, LSE form optimized_c500_flash_attn.cu:666-728) and the
 * split policy (submission_clean.cu:375-430) -- for query-row counts up to 32 per KV head.
 *
 * Layout of the work ("swap AB": key tokens in the MMA M dimension, query rows in N):
 *   S^T[128 tokens, N rows]  = K_tile[128 tokens, 128 d] . Q^T[128 d, N rows]     (TMEM)
 *   O^T[128 d, N rows]      += V_tile^T[128 d, 128 tokens] . P^T[128 tokens, N rows] (TMEM)
 * N = query rows of one KV head (g * Sq) padded to 16 or 32.  A unit is (sequence, KV head).
 *
 * One persistent CTA per SM, 8 warps with fixed roles:
 *   warps 0, 3  TMA producers (warp 0 K, warp 3 V, after allocating TMEM): 16-token page
 *               boxes into rings of 128-token K and V tiles (128-byte swizzle, the layout
 *               the MMA reads as K-major K and MN-major V^T); a K slot is refilled once
 *               QK^T has read it, a V slot once PV (bf16) or the f16 conversion (e4m3) has.
 *   warp 1      MMA issuer (one thread): QK^T of tile i+1 is issued before PV of tile i, so
 *               the softmax of one tile overlaps the tensor core's work on its neighbours.
 *   warp 2      Q loader: a unit's query rows into shared memory (e4m3 pools: q split into
 *               two exact e4m3 terms, hi + lo, with a power-of-two row scale); it also makes
 *               the counter arrival for the slice's first piece when that piece ends
 *               mid-stream, so the softmax warps do not wait for its round trips.
 *   warps 4-7   softmax and epilogue: thread t owns TMEM lane t, i.e. token t of S^T and
 *               dimension t of O^T.  Online softmax in the log2 domain with a lazily moved
 *               reference max (it moves only when a score exceeds it by 2^8; the O^T
 *               columns are then rescaled in TMEM); P^T goes to shared memory as the B
 *               operand of the PV MMA, in bf16 next to bf16 V.  With e4m3 pools thread t
 *               also converts V row t of the tile to f16 (exact) and P is f16: e4m3 P would
 *               lose the small weights (its smallest step is 2^-9, and weights far below
 *               that still matter when |V| is large), so PV runs in kind::f16.
 * The work is cut into equal contiguous slices of 16-token chunks per CTA over the actual
 * lengths (pgqa_partition.h); a unit cut by a slice boundary writes a record (normalised
 * O, log2-sum-exp) and the last CTA to arrive on the unit's counter merges the records.
 *
 * Every wait is bounded; a wait that expires sets the device error word and a CTA-wide
 * abort flag, every role then leaves its loop, the MMA issuer and the producer wait
 * (bounded) for their operations in flight, TMEM is freed and the CTA still arrives on the
 * counters of the units it cuts, so the workspace is left zeroed.
 */
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "pgqa_partition.h"
#include "pgqa_ptx.cuh"
#include "pgqa_tc.h"

namespace pgqa {
namespace tc {

constexpr int kTileChunks = 8;                      // 128 tokens per tile
constexpr int kThreads = 256;
constexpr float kLazyLog2 = 8.f;
enum : int32_t { kErrTimeout = 1, kErrBadPage = 2, kErrBadSeqlen = 4 };

/* K and V tiles stream through separate rings, each filled by its own producer warp: a K
 * slot is free again once QK^T has read it, a V slot once PV has (bf16) or once V has been
 * converted to f16 (e4m3), so neither ring waits for the other's consumer. */
template <bool KV8, int NP>
struct Geo {
    static constexpr int kHalf = 16384;                     // 128 tokens x 128 bytes
    static constexpr int kSlot = KV8 ? kHalf : 2 * kHalf;   // one K or V tile
    static constexpr int kChunkBytes = KV8 ? 2048 : 4096;   // one tensor, 16 tokens
    static constexpr int kSK = KV8 ? (NP <= 16 ? 4 : 3) : (NP <= 16 ? 3 : 2);
    static constexpr int kSV = KV8 ? (NP <= 16 ? 4 : 3) : 3;
};

/* Shared-memory matrix descriptor: start, leading / stride byte offsets, layout type. */
__device__ __forceinline__ uint64_t sdesc(uint32_t addr, uint32_t lbo, uint32_t sbo, uint32_t layout) {
    return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | ((uint64_t)1 << 46) | ((uint64_t)layout << 61);
}
constexpr uint32_t kSw128 = 2, kSwNone = 0;

/* Instruction descriptor: fp32 accumulator, A/B format (bf16 = 1 for kind::f16, e4m3 = 0 for
 * kind::f8f6f4), A/B major (0 = K-major, 1 = MN-major), N, M = 128. */
__host__ __device__ constexpr uint32_t idesc(uint32_t fmt, uint32_t a_mn, uint32_t b_mn, uint32_t n) {
    return (1u << 4) | (fmt << 7) | (fmt << 10) | (a_mn << 15) | (b_mn << 16) | ((n >> 3) << 17) |
           ((128u >> 4) << 24);
}

struct Tile {
    int32_t b, kvh, c0, nc, n, L;  // sequence, KV head, first chunk, chunks, unit chunks, length
    bool first, last;              // first / last tile of this CTA's piece of the unit
};

__device__ __forceinline__ int32_t clamp_len(int64_t L, int64_t cap) {
    return L < 0 ? 0 : (L > cap ? (int32_t)cap : (int32_t)L);
}

/* Largest b with pre[b] * U <= x. */
__device__ __forceinline__ int32_t find_seq(const uint32_t* pre, int32_t B, int64_t U, int64_t x) {
    int32_t lo = 0, hi = B;
    while (hi - lo > 1) {
        const int32_t mid = (lo + hi) >> 1;
        if ((int64_t)pre[mid] * U <= x) lo = mid; else hi = mid;
    }
    return lo;
}

/* Walks a CTA's slice [cs, ce) of flat chunks as tiles of up to 8 chunks; every role runs
 * its own copy, so all roles see the same tile sequence. */
struct Walker {
    const uint32_t* pre;
    int64_t pos, ce;
    int32_t b, j, c, n, L;
    bool piece_start;
    __device__ void init(const TcParams& p, const uint32_t* pre_, int64_t cs, int64_t ce_) {
        pre = pre_;
        pos = cs;
        ce = ce_;
        piece_start = true;
        b = j = c = n = L = 0;
        if (cs < ce) {
            b = find_seq(pre, p.B, p.Hkv, cs);
            n = (int32_t)(pre[b + 1] - pre[b]);
            const int64_t r = cs - (int64_t)pre[b] * p.Hkv;
            j = (r <= kSmallProduct) ? (int32_t)((uint32_t)r / (uint32_t)n) : (int32_t)(r / n);
            c = (int32_t)(r - (int64_t)j * n);
            L = clamp_len((int64_t)__ldg(p.seq_lens + b) + p.len_add, p.cap_tokens);
        }
    }
    __device__ bool next(const TcParams& p, Tile& t) {
        if (pos >= ce) return false;
        int32_t nc = n - c < kTileChunks ? n - c : kTileChunks;
        if (ce - pos < nc) nc = (int32_t)(ce - pos);
        t.b = b; t.kvh = j; t.c0 = c; t.nc = nc; t.n = n; t.L = L;
        t.first = piece_start;
        t.last = (c + nc == n) || (pos + nc == ce);
        pos += nc;
        c += nc;
        piece_start = false;
        if (c == n && pos < ce) {
            c = 0;
            piece_start = true;
            if (++j == p.Hkv) {
                j = 0;
                do { ++b; } while (pre[b + 1] == pre[b]);
                n = (int32_t)(pre[b + 1] - pre[b]);
                L = clamp_len((int64_t)__ldg(p.seq_lens + b) + p.len_add, p.cap_tokens);
            }
        }
        return true;
    }
};

template <bool MQ>
__device__ __forceinline__ int64_t row_offset(const TcParams& p, int32_t b, int32_t kvh, int r) {
    if (!MQ) return ((int64_t)b * p.Hq + kvh * p.g + r) * kHeadDim;
    const int h = r / p.Sq, i = r - (r / p.Sq) * p.Sq;
    return (((int64_t)b * p.Sq + i) * p.Hq + kvh * p.g + h) * kHeadDim;
}

template <bool MQ>
__device__ __forceinline__ int64_t lse_index(const TcParams& p, int32_t b, int32_t kvh, int r) {
    if (!MQ) return (int64_t)b * p.Hq + kvh * p.g + r;
    const int h = r / p.Sq, i = r - (r / p.Sq) * p.Sq;
    return ((int64_t)b * p.Hq + kvh * p.g + h) * p.Sq + i;
}

/* Shared-memory carve-up (offsets from a 1024-byte aligned base). */
template <bool KV8, int NP>
struct Smem {
    static constexpr int SK = Geo<KV8, NP>::kSK;
    static constexpr int SV = Geo<KV8, NP>::kSV;
    static constexpr int kQ = NP * 256;  // bf16: [16 d-chunks][NP rows][16 B]; e4m3: hi, lo [8][NP][16 B]
    static constexpr int kP = NP * 256;  // P^T, 16-bit: [NP/8][128 tokens][16 B]
    static constexpr int kV16 = KV8 ? 2 * Geo<KV8, NP>::kHalf : 0;  // e4m3: V tile as f16 (32 KB)
    static constexpr int kKRing = 0;
    static constexpr int kVRing = kKRing + SK * Geo<KV8, NP>::kSlot;
    static constexpr int kQOff = kVRing + SV * Geo<KV8, NP>::kSlot;
    static constexpr int kPOff = kQOff + 2 * kQ;
    static constexpr int kV16Off = kPOff + 2 * kP;
    static constexpr int kBarOff = kV16Off + 2 * kV16;
    static constexpr int kBars = 2 * SK + 2 * SV + 20;
    static constexpr int kMiscOff = (kBarOff + kBars * 8 + 15) / 16 * 16;
    // misc: [0] TMEM base, [4] abort flag, [8] warp 2's arrival outcome, [16..48) warp sums,
    // [48..80) exchange words
    // [2][4], then red[2][NP][4] f32, mul[2][NP] f32, row offsets and causal masks [NP] each,
    // then the prefix table
    static constexpr int kRedOff = kMiscOff + 80;
    static constexpr int kMulOff = kRedOff + 2 * NP * 4 * 4;
    static constexpr int kRowOff = kMulOff + 2 * NP * 4;   // [NP] row offsets in q / out
    static constexpr int kVisOff = kRowOff + NP * 4;       // [NP] causal visibility masks
    static constexpr int kLPartOff = kVisOff + NP * 4;      // [2][NP][4] per-warp row sums of a piece
    static constexpr int kMRefOff = kLPartOff + 2 * NP * 16; // [2][NP] reference maxima of a piece
    static constexpr int kStgOff = (kMRefOff + 2 * NP * 4 + 15) / 16 * 16;  // epilogue staging
    static constexpr int kStg = NP * kHeadDim * 4;                           // (8 KB at 16 rows or 32)
    static constexpr int kPreOff = kStgOff + (NP == 16 ? kStg : kStg / 2);
    static size_t bytes(int64_t B) { return 1024 + kPreOff + (size_t)(B + 1) * 4 + 16; }
};

template <bool KV8, bool MQ, int NP, bool LSE>
__global__ void __launch_bounds__(kThreads, 1)
pgqa_tc_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
               const TcParams p) {
    using G = Geo<KV8, NP>;
    using L = Smem<KV8, NP>;
    constexpr int SK = G::kSK, SV = G::kSV;
    constexpr int B2 = 2 * SK + 2 * SV;  // first barrier after the ring barriers
    constexpr uint32_t kTmemCols = 4 * NP;  // S^T x2, O^T x2
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (ptx::smem_u32(smem_raw) & 1023u)) & 1023u);
    const uint32_t sb0 = ptx::smem_u32(smem);
    const uint32_t kring = sb0 + L::kKRing;
    const uint32_t vring = sb0 + L::kVRing;
    const uint32_t qbuf = sb0 + L::kQOff;
    const uint32_t pbuf = sb0 + L::kPOff;
    const uint32_t v16buf = sb0 + L::kV16Off;
    const uint32_t bars = sb0 + L::kBarOff;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMiscOff);
    volatile int32_t* abort_flag = reinterpret_cast<volatile int32_t*>(smem + L::kMiscOff + 4);
    // 0: warp 2 did not arrive for the first cut unit, 1: it did, 2: it did and was last
    volatile int32_t* w2flag = reinterpret_cast<volatile int32_t*>(smem + L::kMiscOff + 8);
    int32_t* wsum = reinterpret_cast<int32_t*>(smem + L::kMiscOff + 16);
    volatile int32_t* xword = reinterpret_cast<volatile int32_t*>(smem + L::kMiscOff + 48);  // [2][4]
    float* red = reinterpret_cast<float*>(smem + L::kRedOff);    // [2][NP][4]
    float* mulv = reinterpret_cast<float*>(smem + L::kMulOff);   // [2][NP]
    int32_t* roff = reinterpret_cast<int32_t*>(smem + L::kRowOff);
    uint32_t* vism = reinterpret_cast<uint32_t*>(smem + L::kVisOff);
    float* lpart = reinterpret_cast<float*>(smem + L::kLPartOff);
    float* mrefs = reinterpret_cast<float*>(smem + L::kMRefOff);
    uint8_t* stg = smem + L::kStgOff;  // normalised rows of a piece, [NP][128] (fp32 at 16 rows, bf16 else)
    uint32_t* pre = reinterpret_cast<uint32_t*>(smem + L::kPreOff);

    // barrier addresses
    auto KFULL = [&](int s) { return bars + 8u * s; };
    auto KEMPTY = [&](int s) { return bars + 8u * (SK + s); };
    auto VFULL = [&](int s) { return bars + 8u * (2 * SK + s); };
    auto VEMPTY = [&](int s) { return bars + 8u * (2 * SK + SV + s); };
    auto SFULL = [&](int b) { return bars + 8u * (B2 + b); };
    auto SFREE = [&](int b) { return bars + 8u * (B2 + 2 + b); };
    auto PFULL = [&](int b) { return bars + 8u * (B2 + 4 + b); };
    auto PFREE = [&](int b) { return bars + 8u * (B2 + 6 + b); };
    auto OFULL = [&](int b) { return bars + 8u * (B2 + 8 + b); };
    auto OFREE = [&](int b) { return bars + 8u * (B2 + 10 + b); };
    auto QFULL = [&](int b) { return bars + 8u * (B2 + 12 + b); };
    auto QFREE = [&](int b) { return bars + 8u * (B2 + 14 + b); };
    const uint32_t XG = bars + 8u * (B2 + 16);       // softmax-group exchange
    const uint32_t MMADONE = bars + 8u * (B2 + 17);  // every MMA issued has completed
    const uint32_t RECDONE = bars + 8u * (B2 + 18);  // the slice's first cut record is stored
    const uint32_t W2DONE = bars + 8u * (B2 + 19);   // warp 2 has arrived for it (or given up)

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;

    if (tid == 0) {
        ptx::prefetch_tensormap(&kmap);
        ptx::prefetch_tensormap(&vmap);
        for (int s = 0; s < SK; ++s) {
            ptx::mbar_init(KFULL(s), 1);
            ptx::mbar_init(KEMPTY(s), 1);
        }
        for (int s = 0; s < SV; ++s) {
            ptx::mbar_init(VFULL(s), 1);
            ptx::mbar_init(VEMPTY(s), KV8 ? 4 : 1);  // e4m3: released by the 4 V-converting warps
        }
        for (int b = 0; b < 2; ++b) {
            ptx::mbar_init(SFULL(b), 1);
            // softmax-group barriers take one arrival per warp (after __syncwarp): 128
            // separate arrivals on one shared-memory word serialise
            ptx::mbar_init(SFREE(b), 4);
            ptx::mbar_init(PFULL(b), 4);
            ptx::mbar_init(PFREE(b), 1);
            ptx::mbar_init(OFULL(b), 1);
            ptx::mbar_init(OFREE(b), 4);
            ptx::mbar_init(QFULL(b), 1);
            ptx::mbar_init(QFREE(b), 1 + 4);
        }
        ptx::mbar_init(XG, 4);
        ptx::mbar_init(MMADONE, 1);
        ptx::mbar_init(RECDONE, 4);
        ptx::mbar_init(W2DONE, 1);
        *abort_flag = 0;
        *w2flag = 0;
        ptx::fence_mbar_init();
    }

    // Bounded wait on phase `parity`; gives up at once when another thread has aborted.
    auto wait_bar = [&](uint32_t bar, uint32_t parity) -> bool {
        if (ptx::mbar_try_wait(bar, parity)) return true;
        const uint64_t t0 = ptx::globaltimer_ns();
        for (uint32_t it = 1;; ++it) {
            if (ptx::mbar_try_wait(bar, parity)) return true;
            if ((it & 63u) == 0u) {
                if (*abort_flag) return false;
                if (ptx::globaltimer_ns() - t0 > p.wait_limit_ns) {
                    *abort_flag = 1;
                    atomicOr(p.err, kErrTimeout);
                    return false;
                }
            }
        }
    };
    // Bounded wait that ignores the abort flag (draining operations in flight).
    auto drain_bar = [&](uint32_t bar, uint32_t parity) {
        const uint64_t t0 = ptx::globaltimer_ns();
        while (!ptx::mbar_try_wait(bar, parity)) {
            if (ptx::globaltimer_ns() - t0 > p.wait_limit_ns) {
                atomicOr(p.err, kErrTimeout);
                return;
            }
        }
    };
    // Warp-uniform bounded wait (before warp-collective tcgen05 instructions).
    auto wait_all = [&](uint32_t bar, uint32_t parity) -> bool {
        const bool ok = wait_bar(bar, parity);
        return __all_sync(0xffffffffu, ok);
    };

    if (tid < NP) {
        // row r of a KV head = (head r / Sq, token r % Sq): its offset in q / out relative
        // to (sequence b, KV head kvh), and the rows a key at distance k past
        // L - Sq + 1 stays visible to under the causal mask (bit r set: r % Sq > k).
        // From the parameters alone, so it runs before the wait.
        const int h = MQ ? tid / p.Sq : tid, i = MQ ? tid - (tid / p.Sq) * p.Sq : 0;
        roff[tid] = (i * p.Hq + h) * kHeadDim;
        uint32_t m = 0;
        if (MQ) {
            int rm = 0;  // r % Sq
            for (int r = 0; r < NP; ++r) {
                if (rm > tid) m |= 1u << r;
                if (++rm == p.Sq) rm = 0;
            }
        }
        vism[tid] = m;
    }

    ptx::griddep_wait();
    // The next kernel in the stream may be scheduled from now on: its CTAs take SMs only
    // as this grid's CTAs leave them, and it waits for this grid's completion before it
    // reads memory, so its launch and prologue overlap this grid's tail.
    ptx::griddep_launch_dependents();

    /* ---- chunk prefix over sequences (every CTA; thread tid owns [sb0_, sb1_)) ---- */
    {
        const int per = (p.B + kThreads - 1) / kThreads;
        const int s0 = min(p.B, tid * per), s1 = min(p.B, s0 + per);
        int32_t bad = 0;
        uint32_t local = 0, cmin = 0xffffffffu, cmax = 0;
        for (int b = s0; b < s1; ++b) {
            const int32_t L0 = __ldg(p.seq_lens + b);
            const int64_t Lk = (int64_t)L0 + p.len_add;
            if (L0 < 0 || Lk > p.cap_tokens) bad = 1;
            const uint32_t nb = (uint32_t)seq_chunks(Lk, p.cap_tokens);
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
            wsum[warp] = (int32_t)incl;
            // the warp's common chunk count (-1: its sequences differ, -2: it has none), in
            // the row-maximum buffer, which the softmax warps first use after the TMEM barrier
            reinterpret_cast<int32_t*>(red)[warp] = cmin > cmax ? -2 : (cmin == cmax ? (int32_t)cmin : -1);
        }
        __syncthreads();
        uint32_t run = incl - local;
        for (int w2 = 0; w2 < warp; ++w2) run += (uint32_t)wsum[w2];
        if (tid == kThreads - 1) pre[p.B] = run + local;
        for (int b = s0; b < s1; ++b) {
            pre[b] = run;
            run += (uint32_t)seq_chunks((int64_t)__ldg(p.seq_lens + b) + p.len_add, p.cap_tokens);
        }
        if (bad && blockIdx.x == 0) atomicOr(p.err, kErrBadSeqlen);
        __syncthreads();
    }
    if (blockIdx.x == 0) {  // zero-length sequences produce zeros
        for (int b = tid; b < p.B; b += kThreads) {
            if (pre[b + 1] == pre[b]) {
                uint4* o4 = reinterpret_cast<uint4*>(p.out + (int64_t)b * p.Sq * p.Hq * kHeadDim);
                for (int i = 0; i < p.Sq * p.Hq * kHeadDim / 8; ++i) o4[i] = make_uint4(0, 0, 0, 0);
                if (LSE)
                    for (int i = 0; i < p.Hq * p.Sq; ++i) p.lse_out[(int64_t)b * p.Hq * p.Sq + i] = -INFINITY;
            }
        }
    }
    const int64_t T = (int64_t)pre[p.B] * p.Hkv;
    if (T == 0) return;
    int64_t nct = active_ctas(T, gridDim.x, 1, p.min_chunks);
    if ((int64_t)p.B * p.Hkv <= nct && nct % ((int64_t)p.B * p.Hkv) != 0) {  // equal units: align
        int32_t u = -2;
        bool same = true;
        for (int w2 = 0; w2 < kThreads / 32; ++w2) {
            const int32_t v = reinterpret_cast<const int32_t*>(red)[w2];
            if (v == -1 || (v >= 0 && u >= 0 && v != u)) same = false;
            if (v >= 0) u = v;
        }
        nct = align_ctas(nct, (int64_t)p.B * p.Hkv, same && u > 0);
    }
    if ((int64_t)blockIdx.x >= nct) return;
    const int64_t cs = slice_begin(blockIdx.x, nct, T);
    const int64_t ce = slice_begin(blockIdx.x + 1, nct, T);

    if (warp == 3) {
        ptx::tmem_alloc(ptx::smem_u32(tmem_slot), kTmemCols);
        ptx::tmem_relinquish();
    }
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t tS0 = tmem, tO0 = tmem + 2 * NP;

    if (warp == 0 || warp == 3) {
        /* ================= TMA producers: warp 0 K tiles, warp 3 V tiles ================= */
        const bool isK = (warp == 0);
        const int NS = isK ? SK : SV;
        const uint32_t base = isK ? kring : vring;
        const CUtensorMap* map = isK ? &kmap : &vmap;
        const uint64_t pol = ptx::policy_evict_first();
        Walker w;
        w.init(p, pre, cs, ce);
        Tile t;
        int it = 0;
        int32_t win_b = -1, win_p0 = 0, win_pid = 0;
        const int P = p.page_size;
        auto page_of = [&](int32_t tok) { return p.page_shift >= 0 ? (tok >> p.page_shift) : tok / P; };
        while (w.next(p, t)) {
            const int slot = it % NS;
            const uint32_t empty = isK ? KEMPTY(slot) : VEMPTY(slot);
            if (it >= NS && !wait_bar(empty, ((it / NS) - 1) & 1)) break;
            const int32_t page0 = page_of(t.c0 * kChunkTokens);
            const int32_t pageN = page_of((t.c0 + t.nc - 1) * kChunkTokens);
            if (t.b != win_b || page0 < win_p0 || pageN >= win_p0 + 32) {
                win_b = t.b;
                win_p0 = page0;
                // ceil(L / P) = ceil(16 n / P) (P a multiple of 16): no wait for the length
                const int32_t npg = page_of(t.n * kChunkTokens + P - 1);
                const int32_t pg = page0 + lane;
                win_pid = (pg < npg) ? __ldg(p.block_table + (int64_t)t.b * p.bt_stride + pg) : 0;
            }
            const int k = lane < t.nc ? lane : 0;
            const int32_t tok = (t.c0 + k) * kChunkTokens;
            const int32_t page = page_of(tok);
            int32_t pid = __shfl_sync(0xffffffffu, win_pid, page - win_p0);
            const uint32_t bar = isK ? KFULL(slot) : VFULL(slot);
            if (lane == 0) {
                const uint32_t extra = (isK && p.debug_stuck > 0 && blockIdx.x == 0 && it == 0) ? 16u : 0u;
                ptx::mbar_arrive_expect_tx(bar, (uint32_t)(t.nc * G::kChunkBytes) + extra);
            }
            __syncwarp();
            if (lane < t.nc) {
                if ((uint32_t)pid >= (uint32_t)p.num_pages) {
                    if (isK) atomicOr(p.err, kErrBadPage);
                    pid = 0;
                }
                const int32_t z = pid * P + (tok - page * P);
                const uint32_t dst = base + (uint32_t)slot * G::kSlot + (uint32_t)k * 2048u;
                ptx::tma_load_3d(dst, map, bar, 0, t.kvh, z, pol);
                if (!KV8) ptx::tma_load_3d(dst + G::kHalf, map, bar, 64, t.kvh, z, pol);
            }
            ++it;
        }
        // drain: the loads of the last NS tiles issued may still be in flight
        if (lane == 0)
            for (int k = it > NS ? it - NS : 0; k < it; ++k)
                drain_bar(isK ? KFULL(k % NS) : VFULL(k % NS), (k / NS) & 1);
        __syncwarp();
    } else if (warp == 1) {
        /* ================= MMA issuer (one thread) ================= */
        if (lane == 0) {
            constexpr uint32_t fmt = KV8 ? 0u : 1u;
            constexpr uint32_t id_qk = idesc(fmt, 0, 0, NP);  // A = K (K-major), B = Q (K-major)
            // A = V^T (MN-major), B = P^T (MN-major); e4m3 pools: f16 copies of V and P
            constexpr uint32_t id_pv = idesc(KV8 ? 0u : 1u, 1, 1, NP);
            int pq = -1, po = -1;
            // QK^T of tile i into S buffer i & 1 (its barriers have been checked)
            auto qk = [&](const Tile& t, int i) {
                const int slot = i % SK;
                const int sb = i & 1;
                ptx::tc_fence_after();
                const uint32_t kb = kring + (uint32_t)slot * G::kSlot;
                const uint32_t qb = qbuf + (uint32_t)(pq & 1) * L::kQ;
                const uint32_t d = tS0 + (uint32_t)(sb * NP);
                if (KV8) {
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks) {
                        const uint64_t a = sdesc(kb + ks * 32, 16, 1024, kSw128);
                        const uint64_t bh = sdesc(qb + ks * 2 * NP * 16, NP * 16, 128, kSwNone);
                        const uint64_t bl = sdesc(qb + NP * 128 + ks * 2 * NP * 16, NP * 16, 128, kSwNone);
                        ptx::tc_mma_f8(d, a, bh, id_qk, ks > 0 ? 1u : 0u);
                        ptx::tc_mma_f8(d, a, bl, id_qk, 1u);
                    }
                } else {
#pragma unroll
                    for (int ks = 0; ks < 8; ++ks) {
                        const uint64_t a = sdesc(kb + (ks >> 2) * G::kHalf + (ks & 3) * 32, 16, 1024, kSw128);
                        const uint64_t b = sdesc(qb + ks * 2 * NP * 16, NP * 16, 128, kSwNone);
                        ptx::tc_mma_f16(d, a, b, id_qk, ks > 0 ? 1u : 0u);
                    }
                }
                ptx::tc_commit(SFULL(sb));
                ptx::tc_commit(KEMPTY(slot));
                if (t.last) ptx::tc_commit(QFREE(pq & 1));
            };
            // PV of tile i into O buffer of its piece (its barriers have been checked)
            auto pv = [&](const Tile& t, int i) {
                const int sb = i & 1;
                ptx::tc_fence_after();
                const int vslot = i % SV;
                const uint32_t vb = KV8 ? v16buf + (uint32_t)sb * L::kV16
                                        : vring + (uint32_t)vslot * G::kSlot;
                const uint32_t pb = pbuf + (uint32_t)sb * L::kP;
                const uint32_t d = tO0 + (uint32_t)((po & 1) * NP);
                for (int ks = 0; ks < t.nc; ++ks) {  // 16 tokens per MMA
                    const uint64_t a = sdesc(vb + ks * 2048, G::kHalf, 1024, kSw128);
                    const uint64_t b = sdesc(pb + ks * 256, 128, 2048, kSwNone);
                    ptx::tc_mma_f16(d, a, b, id_pv, (t.first && ks == 0) ? 0u : 1u);
                }
                if (!KV8) ptx::tc_commit(VEMPTY(vslot));
                ptx::tc_commit(PFREE(sb));
                if (t.last) ptx::tc_commit(OFULL(po & 1));
            };
            /* Two queues, served as their operands become ready (non-blocking tests): QK^T
             * runs ahead of the softmax by up to the two S buffers, PV follows each tile's
             * softmax.  Neither waits for the other's inputs. */
            Walker wqk, wpv;
            wqk.init(p, pre, cs, ce);
            wpv.init(p, pre, cs, ce);
            Tile tq, tp;
            bool hq = wqk.next(p, tq), hp = wpv.next(p, tp);
            int iq = 0, ip = 0;
            uint64_t t_idle = 0;
            uint32_t spins = 0;
            while (hp) {
                bool progress = false;
                if (ip < iq) {
                    const int sb = ip & 1;
                    const int pn = po + 1;  // piece of tile ip when it starts one
                    if (ptx::mbar_test_wait(PFULL(sb), (ip >> 1) & 1) &&
                        (KV8 || ptx::mbar_test_wait(VFULL(ip % SV), (ip / SV) & 1)) &&
                        (!tp.first || pn < 2 || ptx::mbar_test_wait(OFREE(pn & 1), ((pn >> 1) - 1) & 1))) {
                        if (tp.first) ++po;
                        pv(tp, ip);
                        ++ip;
                        hp = wpv.next(p, tp);
                        progress = true;
                    }
                }
                if (hq) {
                    const int sb = iq & 1;
                    const int qn = pq + 1;
                    if (ptx::mbar_test_wait(KFULL(iq % SK), (iq / SK) & 1) &&
                        (iq < 2 || ptx::mbar_test_wait(SFREE(sb), ((iq >> 1) - 1) & 1)) &&
                        (!tq.first || ptx::mbar_test_wait(QFULL(qn & 1), (qn >> 1) & 1))) {
                        if (tq.first) ++pq;
                        qk(tq, iq);
                        ++iq;
                        hq = wqk.next(p, tq);
                        progress = true;
                    }
                }
                if (progress) {
                    t_idle = 0;
                    spins = 0;
                    continue;
                }
                // back off: this warp shares its SM sub-partition with a softmax warp
                __nanosleep(20);
                if ((++spins & 15u) == 0u) {
                    if (*abort_flag) break;
                    const uint64_t now = ptx::globaltimer_ns();
                    if (t_idle == 0) {
                        t_idle = now;
                    } else if (now - t_idle > p.wait_limit_ns) {
                        *abort_flag = 1;
                        atomicOr(p.err, kErrTimeout);
                        break;
                    }
                }
            }
            // every MMA issued must be complete before TMEM is freed
            ptx::tc_commit(MMADONE);
            drain_bar(MMADONE, 0);
        }
        __syncwarp();
    } else if (warp == 2) {
        /* ================= Q loader ================= */
        Walker w;
        w.init(p, pre, cs, ce);
        /* The slice's first cut unit, when another piece follows it here: the softmax
         * group stores its record mid-stream (RECDONE) and this warp makes the arrival on
         * the unit's counter (release, atomic; for a last arrival the reset and acquire),
         * so that the stream does not wait for those round trips.  The outcome goes to
         * w2flag and W2DONE, which the softmax group reads after its stream. */
        const int32_t fb = w.b, fj = w.j, fn = w.n;
        const int64_t fbeg = (int64_t)pre[fb] * p.Hkv + (int64_t)fj * fn;
        bool first_pending = (w.c != 0) && (fbeg + fn < ce);
        auto first_arrive = [&](bool got) {
            int32_t f = 0;
            if (got && lane == 0) {
                const int64_t c_first = slice_owner(fbeg, nct, T);
                const int64_t c_last = slice_owner(fbeg + fn - 1, nct, T);
                int32_t* cnt = p.counters + (int64_t)fb * p.Hkv + fj;
                // the record stores, ordered before this thread by RECDONE (cumulative)
                ptx::fence_acq_rel_gpu();
                const int32_t prev = ptx::atom_add_acq_rel_gpu(cnt, 1);
                f = 1;
                if (prev == (int32_t)(c_last - c_first)) {
                    *cnt = 0;
                    ptx::fence_acq_rel_gpu();  // the other CTAs' records, for the merge
                    f = 2;
                }
            }
            if (lane == 0) {
                *w2flag = f;
                ptx::mbar_arrive(W2DONE);
            }
            __syncwarp();
            first_pending = false;
        };
        Tile t;
        int pc = 0;
        while (w.next(p, t)) {
            if (!t.first) continue;
            const int qb = pc & 1;
            // a record handed over since the last look is released before the next wait
            if (first_pending && __shfl_sync(0xffffffffu, lane == 0 && ptx::mbar_test_wait(RECDONE, 0) ? 1 : 0, 0))
                first_arrive(true);
            if (pc >= 2 && !wait_all(QFREE(qb), ((pc >> 1) - 1) & 1)) break;
            const uint32_t qs = qbuf + (uint32_t)qb * L::kQ;
            const int r = lane;
            if (r < NP) {
                const bool valid = r < p.rows;
                float mul = p.scale_log2;
                if (!KV8) {
                    const uint4* src = valid ? reinterpret_cast<const uint4*>(p.q + row_offset<MQ>(p, t.b, t.kvh, r)) : nullptr;
#pragma unroll
                    for (int kc = 0; kc < 16; ++kc) {
                        const uint4 v = valid ? __ldg(src + kc) : make_uint4(0, 0, 0, 0);
                        ptx::sts_u4(qs + (uint32_t)(kc * NP + r) * 16u, v);
                    }
                } else {
                    float x[128];
                    if (valid) {
                        const uint4* src = reinterpret_cast<const uint4*>(p.q + row_offset<MQ>(p, t.b, t.kvh, r));
#pragma unroll
                        for (int kc = 0; kc < 16; ++kc) {
                            const uint4 v = __ldg(src + kc);
                            const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                x[kc * 8 + 2 * e] = __uint_as_float(w4[e] << 16);
                                x[kc * 8 + 2 * e + 1] = __uint_as_float(w4[e] & 0xffff0000u);
                            }
                        }
                    } else {
#pragma unroll
                        for (int i = 0; i < 128; ++i) x[i] = 0.f;
                    }
                    float mx = 0.f;
#pragma unroll
                    for (int i = 0; i < 128; ++i) mx = fmaxf(mx, fabsf(x[i]));
                    // power-of-two row scale: largest |q| * 2^e in [128, 256) (e4m3 max 448)
                    int e = 0;
                    if (mx > 0.f) e = 7 - ((int)((__float_as_uint(mx) >> 23) & 0xff) - 127);
                    e = max(-100, min(100, e));
                    const float up = exp2f((float)e);
                    const float ks = (p.k_scale != nullptr) ? __ldg(p.k_scale + t.kvh) : 1.f;
                    mul = p.scale_log2 * ks * exp2f((float)-e);
#pragma unroll
                    for (int kc = 0; kc < 8; ++kc) {  // 16 dims per 16-byte row of a core matrix
                        uint32_t hi[4], lo[4];
#pragma unroll
                        for (int q4 = 0; q4 < 4; ++q4) {
                            const int i0 = kc * 16 + q4 * 4;
                            const float a0 = x[i0] * up, a1 = x[i0 + 1] * up, a2 = x[i0 + 2] * up, a3 = x[i0 + 3] * up;
                            const uint32_t h01 = ptx::f32x2_to_e4m3x2(a0, a1);
                            const uint32_t h23 = ptx::f32x2_to_e4m3x2(a2, a3);
                            const float2 f01 = ptx::e4m3x2_to_f32x2(h01);
                            const float2 f23 = ptx::e4m3x2_to_f32x2(h23);
                            const uint32_t l01 = ptx::f32x2_to_e4m3x2(a0 - f01.x, a1 - f01.y);
                            const uint32_t l23 = ptx::f32x2_to_e4m3x2(a2 - f23.x, a3 - f23.y);
                            hi[q4] = h01 | (h23 << 16);
                            lo[q4] = l01 | (l23 << 16);
                        }
                        ptx::sts_u4(qs + (uint32_t)(kc * NP + r) * 16u, make_uint4(hi[0], hi[1], hi[2], hi[3]));
                        ptx::sts_u4(qs + NP * 128 + (uint32_t)(kc * NP + r) * 16u, make_uint4(lo[0], lo[1], lo[2], lo[3]));
                    }
                }
                mulv[qb * NP + r] = mul;
            }
            ptx::fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive(QFULL(qb));
            ++pc;
        }
        if (first_pending) first_arrive(wait_all(RECDONE, 0));  // gives up only on an abort
    } else if (warp >= 4) {
        /* ================= softmax and epilogue (128 threads) ================= */
        const int st = tid - 128;          // TMEM lane: token (S^T) / dimension (O^T)
        const int wq = st >> 5;
        const uint32_t lane_off = (uint32_t)(wq * 32) << 16;
        uint32_t xg_n = 0;                 // uses of the exchange barrier so far
        // exchange: every thread arrives, then waits (bounded); data at parity xg_n & 1
        auto xsync = [&]() -> bool {
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive(XG);
            const bool ok = wait_all(XG, xg_n & 1);
            ++xg_n;
            return ok;
        };
        // TMEM loads of NP columns of this thread's lane
        auto tld = [&](uint32_t col, float (&v)[NP]) {
            if (NP == 16) {
                ptx::tc_ld16(col | lane_off, *reinterpret_cast<float(*)[16]>(&v[0]));
            } else {
                ptx::tc_ld16(col | lane_off, *reinterpret_cast<float(*)[16]>(&v[0]));
                ptx::tc_ld16((col + 16) | lane_off, *reinterpret_cast<float(*)[16]>(&v[16]));
            }
        };
        auto tst = [&](uint32_t col, const float (&v)[NP]) {
            ptx::tc_st16(col | lane_off, *reinterpret_cast<const float(*)[16]>(&v[0]));
            if (NP == 32) ptx::tc_st16((col + 16) | lane_off, *reinterpret_cast<const float(*)[16]>(&v[16]));
        };

        float m_ref[NP], l_part[NP];
        float mul[KV8 ? NP : 1];  // bf16: one score multiplier for every row
        float vsc = 1.f;
        int32_t causal_base = 0;  // keys past L - Sq + 1 are seen by some rows only
        int32_t piece_c0 = 0;
        bool done_cut_first = false, done_cut_last = false;
        // cut units of this slice: the one holding chunk cs (if it starts before cs) and
        // the one holding chunk ce-1 (if it ends after ce)
        Walker w;
        w.init(p, pre, cs, ce);
        const bool cut_first = (w.c != 0);
        int32_t last_b, last_j;
        bool cut_last;
        {
            const int32_t bl = find_seq(pre, p.B, p.Hkv, ce - 1);
            const int32_t nl = (int32_t)(pre[bl + 1] - pre[bl]);
            const int64_t rl = ce - 1 - (int64_t)pre[bl] * p.Hkv;
            const int32_t jl = (rl <= kSmallProduct) ? (int32_t)((uint32_t)rl / (uint32_t)nl) : (int32_t)(rl / nl);
            const int32_t cl = (int32_t)(rl - (int64_t)jl * nl);
            last_b = bl;
            last_j = jl;
            cut_last = (cl != nl - 1) && !(bl == w.b && jl == w.j && cut_first);
        }
        const int32_t first_b = w.b, first_j = w.j;

        // record, arrival and (for the last arriver) merge of a unit cut by slice bounds
        // (`arrived` is set once this CTA's arrival on the counter is certain)
        // the normalised row and its log2-sum-exp from O, the row sum l and the reference
        auto norm_of = [&](float o, float l, float vs) { return (!MQ || l > 0.f) ? o * __fdividef(vs, l) : 0.f; };
        auto lse2_of = [&](float m, float l) { return (!MQ || l > 0.f) ? m + ptx::lg2(l) : -INFINITY; };
        // record slot of this CTA for the unit (b, kvh) of n chunks
        auto slot_of = [&](int32_t b, int32_t kvh, int32_t n) {
            return record_slot(blockIdx.x, cs, (int64_t)pre[b] * p.Hkv + (int64_t)kvh * n);
        };
        // record row r (thread st writes dimension st)
        auto put_rec = [&](int64_t slot, int r, float v) {
            if (NP == 16) reinterpret_cast<float*>(p.rec_o)[(slot * NP + r) * kHeadDim + st] = v;
            else reinterpret_cast<__nv_bfloat16*>(p.rec_o)[(slot * NP + r) * kHeadDim + st] = __float2bfloat16_rn(v);
        };
        // bit 0 / 1: this CTA arrived last on the slice's first / last cut unit (their
        // records are merged after the stream); bit 2: the first one went to warp 2
        uint32_t mg_mask = 0;
        // arrival on the counter of a cut unit whose record this CTA has written; the last
        // CTA to arrive queues the unit's merge
        auto arrive_merge = [&](int32_t b, int32_t kvh, int32_t n, bool live, bool& arrived,
                                uint32_t bit) -> bool {
            const int64_t ubeg = (int64_t)pre[b] * p.Hkv + (int64_t)kvh * n;
            const int64_t c_first = slice_owner(ubeg, nct, T);
            const int64_t c_last = slice_owner(ubeg + n - 1, nct, T);
            int32_t* cnt = p.counters + (int64_t)b * p.Hkv + kvh;
            if (!live) {
                // abort path: one thread arrives; a last arriver only resets the counter
                if (st == 0) {
                    const int32_t prev = ptx::atom_add_acq_rel_gpu(cnt, 1);
                    if (prev == (int32_t)(c_last - c_first)) *cnt = 0;
                }
                arrived = true;
                return true;
            }
            if (!xsync()) return false;
            arrived = true;  // thread 0 arrives now, whatever happens next
            if (st == 0) {
                // releases the record stores of all 128 threads, ordered before this
                // thread by the exchange barrier (cumulative release)
                ptx::fence_acq_rel_gpu();
                const int32_t prev = ptx::atom_add_acq_rel_gpu(cnt, 1);
                const int last = prev == (int32_t)(c_last - c_first);
                if (last) {
                    *cnt = 0;
                    ptx::fence_acq_rel_gpu();  // the other CTAs' records, for every thread here
                }
                xword[(xg_n & 1) * 4] = last;
            }
            if (!xsync()) return false;
            if (xword[((xg_n - 1) & 1) * 4]) mg_mask |= bit;  // last: merge after the stream
            return true;
        };
        // merge of every CTA's record of the unit (b, kvh) of n chunks, by the last arriver
        auto merge_records = [&](int32_t b, int32_t kvh, int32_t n) {
            const int64_t ubeg = (int64_t)pre[b] * p.Hkv + (int64_t)kvh * n;
            const int64_t c_first = slice_owner(ubeg, nct, T);
            const int64_t c_last = slice_owner(ubeg + n - 1, nct, T);
            /* Merge the unit's records.  Thread st owns dims [8 dc, 8 dc + 8) of rows
             * [kR rg, kR rg + kR) (dc = st % 16, rg = st / 16), so every load is a 16-byte
             * vector; records are read kB at a time, all loads of a batch in flight
             * together, with the running maxima raised once per batch. */
            constexpr int kR = NP / 8;  // rows per thread
            constexpr int kB = 4;       // records per batch
            const int dc = st & 15, rg = st >> 4;
            const int nrec = (int)(c_last - c_first + 1);
            const int64_t slot0 = record_slot(c_first, slice_begin(c_first, nct, T), ubeg);
            float mx[kR], den[kR], acc[kR][8];
#pragma unroll
            for (int r = 0; r < kR; ++r) {
                mx[r] = -INFINITY;
                den[r] = 0.f;
#pragma unroll
                for (int e = 0; e < 8; ++e) acc[r][e] = 0.f;
            }
            for (int k0 = 0; k0 < nrec; k0 += kB) {
                float lv[kB][kR];
                uint4 ov[kB][kR][NP == 16 ? 2 : 1];
#pragma unroll
                for (int u = 0; u < kB; ++u) {
                    const bool in = k0 + u < nrec;
                    const int64_t sl = (k0 + u == 0) ? slot0 : 2 * (c_first + k0 + u);
#pragma unroll
                    for (int r = 0; r < kR; ++r) {
                        const int row = rg * kR + r;
                        lv[u][r] = in ? __ldcg(p.rec_lse + sl * NP + row) : -INFINITY;
                        if (NP == 16) {
                            const uint4* src = reinterpret_cast<const uint4*>(
                                reinterpret_cast<const float*>(p.rec_o) + (sl * NP + row) * kHeadDim + dc * 8);
                            ov[u][r][0] = in ? __ldcg(src) : make_uint4(0, 0, 0, 0);
                            ov[u][r][NP == 16 ? 1 : 0] = in ? __ldcg(src + 1) : make_uint4(0, 0, 0, 0);
                        } else {
                            const uint4* src = reinterpret_cast<const uint4*>(
                                reinterpret_cast<const __nv_bfloat16*>(p.rec_o) + (sl * NP + row) * kHeadDim + dc * 8);
                            ov[u][r][0] = in ? __ldcg(src) : make_uint4(0, 0, 0, 0);
                        }
                    }
                }
#pragma unroll
                for (int r = 0; r < kR; ++r) {
                    float bm = lv[0][r];
#pragma unroll
                    for (int u = 1; u < kB; ++u) bm = fmaxf(bm, lv[u][r]);
                    if (bm > mx[r]) {  // raise the running maximum, rescaling what was summed
                        const float sc = (mx[r] == -INFINITY) ? 0.f : ptx::ex2(mx[r] - bm);
                        den[r] *= sc;
#pragma unroll
                        for (int e = 0; e < 8; ++e) acc[r][e] *= sc;
                        mx[r] = bm;
                    }
                    const float base = (MQ && mx[r] == -INFINITY) ? 0.f : mx[r];  // no key: weight 0
#pragma unroll
                    for (int u = 0; u < kB; ++u) {
                        const float wgt = ptx::ex2(lv[u][r] - base);
                        den[r] += wgt;
                        float f[8];
                        if (NP == 16) {
                            const uint4 a = ov[u][r][0], c = ov[u][r][NP == 16 ? 1 : 0];
                            f[0] = __uint_as_float(a.x); f[1] = __uint_as_float(a.y);
                            f[2] = __uint_as_float(a.z); f[3] = __uint_as_float(a.w);
                            f[4] = __uint_as_float(c.x); f[5] = __uint_as_float(c.y);
                            f[6] = __uint_as_float(c.z); f[7] = __uint_as_float(c.w);
                        } else {
                            const uint4 a = ov[u][r][0];
                            const uint32_t wv[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                f[2 * e] = __uint_as_float(wv[e] << 16);
                                f[2 * e + 1] = __uint_as_float(wv[e] & 0xffff0000u);
                            }
                        }
#pragma unroll
                        for (int e = 0; e < 8; ++e) acc[r][e] = fmaf(wgt, f[e], acc[r][e]);
                    }
                }
            }
#pragma unroll
            for (int r = 0; r < kR; ++r) {
                const int row = rg * kR + r;
                if (row < p.rows) {
                    const float inv = (!MQ || den[r] > 0.f) ? __fdividef(1.f, den[r]) : 0.f;
                    uint4 o8;
                    o8.x = ptx::pack_bf16x2(acc[r][0] * inv, acc[r][1] * inv);
                    o8.y = ptx::pack_bf16x2(acc[r][2] * inv, acc[r][3] * inv);
                    o8.z = ptx::pack_bf16x2(acc[r][4] * inv, acc[r][5] * inv);
                    o8.w = ptx::pack_bf16x2(acc[r][6] * inv, acc[r][7] * inv);
                    *reinterpret_cast<uint4*>(p.out + ((int64_t)b * p.Sq * p.Hq + (int64_t)kvh * p.g) * kHeadDim +
                                              roff[row] + dc * 8) = o8;
                    if (LSE && dc == 0)
                        p.lse_out[((int64_t)b * p.Hq + (int64_t)kvh * p.g) * p.Sq + row] =
                            (den[r] > 0.f ? mx[r] + ptx::lg2(den[r]) : -INFINITY) * 0.6931471805599453f;
                }
            }
        };


        struct Pending {
            int pc = -1;
            int32_t b = 0, kvh = 0, n = 0;
            float vsc = 1.f;
            bool whole = false, is_first = false;
        } pend;
        // epilogue of piece P: O^T out of TMEM, row sums and maxima from shared memory,
        // then the output rows (a whole unit) or a record and the arrival (a cut unit)
        // handoff: a cut first piece ending mid-stream leaves its arrival to warp 2
        auto epilogue = [&](const Pending& P, bool handoff) -> bool {
            const int ob = P.pc & 1;
            if (!wait_all(OFULL(ob), (P.pc >> 1) & 1)) return false;
            ptx::tc_fence_after();
            const float* lp = lpart + ob * NP * 4;
            const float* mp = mrefs + ob * NP;
            auto lsum_of = [&](int r) {
                const float4 l4 = ptx::lds_f4(ptx::smem_u32(lp + r * 4));
                return (l4.x + l4.y) + (l4.z + l4.w);
            };
            const int64_t slot = P.whole ? 0 : slot_of(P.b, P.kvh, P.n);
            // 16-bit rows for the output and for 32-row records, fp32 for 16-row records
            const bool f32 = !P.whole && NP == 16;
            // O^T streamed 16 columns (rows) at a time into the staging buffer
#pragma unroll
            for (int h = 0; h < NP / 16; ++h) {
                float o16[16];
                ptx::tc_ld16((tO0 + (uint32_t)(ob * NP + 16 * h)) | lane_off, o16);
                ptx::tc_wait_ld();
#pragma unroll
                for (int r16 = 0; r16 < 16; ++r16) {
                    const int r = 16 * h + r16;
                    const float v = norm_of(o16[r16], lsum_of(r), P.vsc);
                    if (f32) reinterpret_cast<float*>(stg)[r * kHeadDim + st] = v;
                    else reinterpret_cast<__nv_bfloat16*>(stg)[r * kHeadDim + st] = __float2bfloat16_rn(v);
                }
            }
            ptx::tc_fence_before();
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive(OFREE(ob));
            // log2-sum-exp of row st (threads st < NP)
            if (st < NP) {
                const float l2 = lse2_of(mp[st], lsum_of(st));
                if (!P.whole) p.rec_lse[slot * NP + st] = l2;
                else if (LSE && st < p.rows)
                    p.lse_out[((int64_t)P.b * p.Hq + (int64_t)P.kvh * p.g) * p.Sq + st] = l2 * 0.6931471805599453f;
            }
            if (!xsync()) return false;
            // the staged rows leave in 16-byte pieces
            const uint4* s4 = reinterpret_cast<const uint4*>(stg);
            if (P.whole) {
                __nv_bfloat16* obase = p.out + ((int64_t)P.b * p.Sq * p.Hq + (int64_t)P.kvh * p.g) * kHeadDim;
                for (int k = st; k < NP * 16; k += 128) {
                    const int r = k >> 4, c = k & 15;
                    if (r < p.rows) *reinterpret_cast<uint4*>(obase + roff[r] + c * 8) = s4[k];
                }
            } else {
                uint4* d4 = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(p.rec_o) +
                                                     slot * (f32 ? NP * kHeadDim * 4 : NP * kHeadDim * 2));
                for (int k = st; k < (f32 ? NP * 32 : NP * 16); k += 128) d4[k] = s4[k];
            }
            if (P.whole) return true;
            if (handoff && P.is_first) {
                // warp 2 takes the release and the arrival (two round trips the stream would
                // otherwise wait for); one arrival per warp after its record stores
                __syncwarp();
                if (lane == 0) ptx::mbar_arrive(RECDONE);
                mg_mask |= 4u;
                return true;
            }
            return arrive_merge(P.b, P.kvh, P.n, true, P.is_first ? done_cut_first : done_cut_last,
                                P.is_first ? 1u : 2u);
        };

        Tile t;
        int i = 0, pc = -1;
        bool ok = true;
        while (ok && w.next(p, t)) {
            const int sb = i & 1;
            if (t.first) {
                ++pc;
                const int qb = pc & 1;
                if (!wait_all(QFULL(qb), (pc >> 1) & 1)) { ok = false; break; }
#pragma unroll
                for (int r = 0; r < (KV8 ? NP : 1); ++r) mul[r] = mulv[qb * NP + r];
                __syncwarp();
                if (lane == 0) ptx::mbar_arrive(QFREE(qb));
#pragma unroll
                for (int r = 0; r < NP; ++r) { m_ref[r] = -INFINITY; l_part[r] = 0.f; }
                if (KV8) vsc = (p.v_scale != nullptr) ? __ldg(p.v_scale + t.kvh) : 1.f;
                causal_base = t.L - p.Sq + 1;
                piece_c0 = t.c0;
            }
            const int32_t tok0 = t.c0 * kChunkTokens;
            const int32_t nvalid = min(t.nc * kChunkTokens, t.L - tok0);
            const int32_t pos = tok0 + st;
            if (!wait_all(SFULL(sb), (i >> 1) & 1)) { ok = false; break; }
            ptx::tc_fence_after();
            float s[NP];
            tld(tS0 + (uint32_t)(sb * NP), s);  // completes at tc_wait_ld below
            if (KV8) {
                /* This thread's V row (token st) from e4m3 to f16, into the swizzled f16 tile
                 * the PV MMA reads (rows past the valid tokens become zeros); the e4m3 stage
                 * is then released to the producer. */
                const int vslot = i % SV;
                if (!wait_all(VFULL(vslot), (i / SV) & 1)) { ok = false; break; }
                if (i >= 2 && !wait_all(PFREE(sb), ((i >> 1) - 1) & 1)) { ok = false; break; }
                if (st < t.nc * kChunkTokens) {
                    const uint32_t src = vring + (uint32_t)(vslot * G::kSlot + st * 128);
                    const uint32_t dst = v16buf + (uint32_t)(sb * L::kV16 + st * 128);
                    const uint32_t sw = (uint32_t)(st & 7);
                    const bool valid = st < nvalid;
#pragma unroll
                    for (int c = 0; c < 8; ++c) {  // 16 dims per 16-byte chunk
                        uint4 w8 = make_uint4(0, 0, 0, 0);
                        if (valid) w8 = ptx::lds_u4(src + (((uint32_t)c ^ sw) << 4));
                        uint32_t h[8];
                        ptx::e4m3x4_to_f16(w8.x, h[0], h[1]);
                        ptx::e4m3x4_to_f16(w8.y, h[2], h[3]);
                        ptx::e4m3x4_to_f16(w8.z, h[4], h[5]);
                        ptx::e4m3x4_to_f16(w8.w, h[6], h[7]);
                        const uint32_t hb = dst + (uint32_t)((c >> 2) * G::kHalf);
                        const uint32_t cc = (uint32_t)(2 * (c & 3));
                        ptx::sts_u4(hb + ((cc ^ sw) << 4), make_uint4(h[0], h[1], h[2], h[3]));
                        ptx::sts_u4(hb + (((cc + 1) ^ sw) << 4), make_uint4(h[4], h[5], h[6], h[7]));
                    }
                }
                __syncwarp();
                if (lane == 0) ptx::mbar_arrive(VEMPTY(vslot));
            }
            ptx::tc_wait_ld();
            ptx::tc_fence_before();
            __syncwarp();
                if (lane == 0) ptx::mbar_arrive(SFREE(sb));

            bool vote = false;
            uint32_t vmask = st < nvalid ? 0xffffffffu : 0u;  // rows that see this key
            if (MQ && p.causal) {
                const int32_t k = pos - causal_base;
                if (k >= 0) vmask = (st < nvalid && k < p.Sq - 1) ? vism[k] : 0u;
            }
#pragma unroll
            for (int r = 0; r < NP; ++r) {
                const bool vis = (vmask >> r) & 1u;
                const float x = vis ? s[r] * mul[KV8 ? r : 0] : -INFINITY;
                s[r] = x;
                vote = vote || (x > m_ref[r] + kLazyLog2);
            }
            // any thread's score beyond its row's reference (+2^8)?  One word per warp.
            {
                const int wv = __any_sync(0xffffffffu, vote) ? 1 : 0;
                if (lane == 0) xword[(xg_n & 1) * 4 + wq] = wv;
            }
            if (!xsync()) { ok = false; break; }
            const int xb = ((xg_n - 1) & 1) * 4;
            const bool voted = (xword[xb] | xword[xb + 1] | xword[xb + 2] | xword[xb + 3]) != 0;
            if (voted) {
                // per-row maxima over the 128 tokens of the tile
                float* rb = red + (xg_n & 1) * NP * 4;
#pragma unroll
                for (int r = 0; r < NP; ++r) {
                    float v = s[r];
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
                    if (lane == 0) rb[r * 4 + wq] = v;
                }
                if (!xsync()) { ok = false; break; }
                float alpha[NP];
#pragma unroll
                for (int r = 0; r < NP; ++r) {
                    const float4 m4 = ptx::lds_f4(ptx::smem_u32(rb + r * 4));
                    const float tm = fmaxf(fmaxf(m4.x, m4.y), fmaxf(m4.z, m4.w));
                    const float mn = fmaxf(m_ref[r], tm);
                    const float z = (MQ && mn == -INFINITY) ? 0.f : mn;
                    alpha[r] = ptx::ex2(m_ref[r] - z);
                    m_ref[r] = mn;
                    l_part[r] *= alpha[r];
                }
                if (!t.first) {
                    // O^T holds this piece's earlier tiles: wait for PV of tile i-1, rescale
                    if (!wait_all(PFREE((i - 1) & 1), ((i - 1) >> 1) & 1)) { ok = false; break; }
                    ptx::tc_fence_after();
                    float o[NP];
                    const uint32_t oc = tO0 + (uint32_t)((pc & 1) * NP);
                    tld(oc, o);
                    ptx::tc_wait_ld();
#pragma unroll
                    for (int r = 0; r < NP; ++r) o[r] *= alpha[r];
                    tst(oc, o);
                    ptx::tc_wait_st();
                }
            }
            float pv[NP];
#pragma unroll
            for (int r = 0; r < NP; ++r) {
                const float base = (MQ && m_ref[r] == -INFINITY) ? 0.f : m_ref[r];
                pv[r] = ptx::ex2(s[r] - base);
                l_part[r] += pv[r];
            }
            if (!KV8 && i >= 2 && !wait_all(PFREE(sb), ((i >> 1) - 1) & 1)) { ok = false; break; }
            // P^T row st, 16-bit (f16 next to the f16 copy of e4m3 V, bf16 next to bf16 V)
            const uint32_t pb = pbuf + (uint32_t)sb * L::kP;
#pragma unroll
            for (int nb = 0; nb < NP / 8; ++nb) {
                const int r0 = nb * 8;
                uint32_t w4[4];
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    w4[k] = KV8 ? ptx::pack_f16x2(pv[r0 + 2 * k], pv[r0 + 2 * k + 1])
                                : ptx::pack_bf16x2(pv[r0 + 2 * k], pv[r0 + 2 * k + 1]);
                ptx::sts_u4(pb + (uint32_t)(nb * 2048 + st * 16), make_uint4(w4[0], w4[1], w4[2], w4[3]));
            }
            // bf16 pools: V rows of tokens past the valid ones inside the last PV step are
            // zeroed in the stage, so that p = 0 never meets a non-finite value left there
            // (e4m3 pools wrote zeros into the f16 copy above)
            if (!KV8 && nvalid < t.nc * kChunkTokens &&
                !wait_all(VFULL(i % SV), (i / SV) & 1)) { ok = false; break; }
            if (!KV8 && st >= nvalid && st < t.nc * kChunkTokens) {
                const uint32_t vrow = vring + (uint32_t)((i % SV) * G::kSlot + st * 128);
#pragma unroll
                for (int c16 = 0; c16 < 8; ++c16) {
                    ptx::sts_u4(vrow + c16 * 16, make_uint4(0, 0, 0, 0));
                    ptx::sts_u4(vrow + G::kHalf + c16 * 16, make_uint4(0, 0, 0, 0));
                }
            }
            ptx::fence_proxy_async_smem();
            ptx::tc_fence_before();
            __syncwarp();
                if (lane == 0) ptx::mbar_arrive(PFULL(sb));

            if (t.last) {
                /* ---- end of this CTA's piece of the unit: its per-warp row sums and its
                 * reference maxima go to shared memory and its epilogue waits one tile (its
                 * O^T buffer stays untouched until the piece after next), so the stream does
                 * not stop for O^T to complete at every unit boundary ---- */
                float* lp = lpart + (pc & 1) * NP * 4;
#pragma unroll
                for (int r = 0; r < NP; ++r) {
                    float v = l_part[r];
#pragma unroll
                    for (int o2 = 16; o2 > 0; o2 >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o2);
                    if (lane == 0) lp[r * 4 + wq] = v;
                }
                if (st == 0)
#pragma unroll
                    for (int r = 0; r < NP; ++r) mrefs[(pc & 1) * NP + r] = m_ref[r];
                Pending nx;
                nx.pc = pc;
                nx.b = t.b;
                nx.kvh = t.kvh;
                nx.n = t.n;
                nx.vsc = vsc;
                nx.whole = (piece_c0 == 0) && (t.c0 + t.nc == t.n);
                nx.is_first = cut_first && t.b == first_b && t.kvh == first_j && piece_c0 != 0;
                // a piece still pending here had only this one tile after it
                if (pend.pc >= 0 && !epilogue(pend, true)) { ok = false; break; }
                pend = nx;
            } else if (pend.pc >= 0 && pend.pc < pc) {
                // one tile after a piece ended (its partials were stored before this tile's
                // exchange, its last PV has long been issued): its epilogue runs now
                if (!epilogue(pend, true)) { ok = false; break; }
                pend.pc = -1;
            }
            ++i;
        }
        if (ok && pend.pc >= 0) {
            // the last piece's partials become visible to every warp at this exchange
            ok = xsync() && epilogue(pend, false);
        }
        if (mg_mask & 4u) {
            // warp 2's arrival for the first cut unit (it arrives on W2DONE in every case)
            drain_bar(W2DONE, 0);
            __syncwarp();
            const int32_t f = *w2flag;
            if (f == 0) {
                // it gave up (the call is aborting): arrive here so the counter is reset
                arrive_merge(first_b, first_j, (int32_t)(pre[first_b + 1] - pre[first_b]), false, done_cut_first, 0u);
            } else {
                done_cut_first = true;
                if (f == 2) mg_mask |= 1u;
            }
        }
        // one call site for the merge code (at most two units: the slice's cut ones)
        for (int k = 0; ok && k < 2; ++k) {
            if (!((mg_mask >> k) & 1u)) continue;
            const int32_t b = k == 0 ? first_b : last_b, kvh = k == 0 ? first_j : last_j;
            merge_records(b, kvh, (int32_t)(pre[b + 1] - pre[b]));
        }
        if (!ok) {
            // a wait expired: still arrive on the counters of the units this slice cuts
            auto empty_record = [&](int32_t b, int32_t kvh, int32_t n) {
                const int64_t slot = slot_of(b, kvh, n);
                for (int r = 0; r < NP; ++r) put_rec(slot, r, 0.f);
                if (st < NP) p.rec_lse[slot * NP + st] = -INFINITY;
            };
            if (cut_first && !done_cut_first) {
                const int32_t n = (int32_t)(pre[first_b + 1] - pre[first_b]);
                empty_record(first_b, first_j, n);
                arrive_merge(first_b, first_j, n, false, done_cut_first, 0u);
            }
            if (cut_last && !done_cut_last) {
                const int32_t n = (int32_t)(pre[last_b + 1] - pre[last_b]);
                empty_record(last_b, last_j, n);
                arrive_merge(last_b, last_j, n, false, done_cut_last, 0u);
            }
        }
    }

    ptx::tc_fence_before();
    __syncthreads();
    if (warp == 3) {
        ptx::tc_fence_after();
        ptx::tmem_dealloc(tmem, kTmemCols);
    }
}

template <bool KV8, bool MQ, int NP, bool LSE>
cudaError_t launch_one(const CUtensorMap& km, const CUtensorMap& vm, const TcParams& p, int grid,
                       size_t smem, bool pdl, cudaStream_t stream) {
    auto kern = pgqa_tc_kernel<KV8, MQ, NP, LSE>;
    static size_t configured[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && configured[dev] < smem) {
        const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        configured[dev] = smem;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, km, vm, p);
}

template <bool KV8, bool MQ, int NP>
cudaError_t launch_lse(const CUtensorMap& km, const CUtensorMap& vm, const TcParams& p, int grid,
                       size_t smem, bool pdl, cudaStream_t stream) {
    return p.lse_out ? launch_one<KV8, MQ, NP, true>(km, vm, p, grid, smem, pdl, stream)
                     : launch_one<KV8, MQ, NP, false>(km, vm, p, grid, smem, pdl, stream);
}

template <bool KV8, bool MQ>
cudaError_t launch_np(const CUtensorMap& km, const CUtensorMap& vm, const TcParams& p, int grid,
                      size_t smem, bool pdl, cudaStream_t stream) {
    return p.rows <= 16 ? launch_lse<KV8, MQ, 16>(km, vm, p, grid, smem, pdl, stream)
                        : launch_lse<KV8, MQ, 32>(km, vm, p, grid, smem, pdl, stream);
}

}  // namespace tc

size_t tc_smem_bytes(bool kv8, int rows, int64_t B) {
    if (rows <= 16) return kv8 ? tc::Smem<true, 16>::bytes(B) : tc::Smem<false, 16>::bytes(B);
    return kv8 ? tc::Smem<true, 32>::bytes(B) : tc::Smem<false, 32>::bytes(B);
}

cudaError_t launch_tc(const CUtensorMap& kmap, const CUtensorMap& vmap, const TcParams& p, bool kv8,
                      int grid, size_t smem, bool pdl, cudaStream_t stream) {
    if (kv8)
        return p.Sq > 1 ? tc::launch_np<true, true>(kmap, vmap, p, grid, smem, pdl, stream)
                        : tc::launch_np<true, false>(kmap, vmap, p, grid, smem, pdl, stream);
    return p.Sq > 1 ? tc::launch_np<false, true>(kmap, vmap, p, grid, smem, pdl, stream)
                    : tc::launch_np<false, false>(kmap, vmap, p, grid, smem, pdl, stream);
}

}  // namespace pgqa
