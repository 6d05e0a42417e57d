// Single-query GQA decode attention over an fp16 / INT8-per-token / INT4-KIVI
// KV cache for sm_100a, with the dequantization fused into a split-sequence
// (FlashDecoding) loop and the log-sum-exp combine fused into the same launch.
//
// Work decomposition
//   unit  = (batch, kv_head, head block): HB query heads that share one KV
//           slab (HB = the GQA group, or a divisor of it), so every KV byte is
//           read from HBM exactly once per step (the reference launches one
//           CTA per query head and re-reads each slab G times, relying on L2).
//   tile  = T consecutive KV positions of one unit (T * row bytes = 32 KB).
//   The flattened (unit, tile) sequence is split evenly over a persistent grid
//   of one CTA per SM: CTA c owns tiles [c*TT/C, (c+1)*TT/C). A CTA's range may
//   cover whole units (written straight to `out`) and partial units at its
//   two ends (written as an un-normalised partial to the workspace; the CTA
//   that completes a unit's last partial, found with an atomic ticket, merges
//   them). No CTA ever waits for another CTA.
//
// Inside a CTA
//   warp 8 (producer): one lane issues 1-D bulk async copies
//     (cp.async.bulk, no tensor map, no multicast) of the K and V tile plus the
//     per-token / per-group scales into an NST-deep shared-memory ring, each
//     stage tracked by a "full" mbarrier with transaction bytes and an "empty"
//     mbarrier the consumers arrive on.
//   warps 0-7 (consumers): warp w owns positions [w*T/8, (w+1)*T/8) of every
//     tile and keeps its own online-softmax state (m, l, acc) for all HB heads,
//     so the tile loop has no CTA-wide barrier. Per warp and tile:
//       QK : 8 lanes per position, 16 channels per lane. K codes are
//            dequantized to fp16 exactly as the reference oracle does
//            (fp16(code * scale [+ zero]); the INT8 token scale multiplies
//            the reduced score instead), then multiplied with q in fp16 by
//            sm_100's mixed-precision fma.rn.f32.f16 (exact product, fp32
//            sum). Partial sums are reduce-scattered over the 8 lanes so each
//            lane ends with one head's score.
//       softmax: scores are in the log2 domain (q pre-scaled by
//            softmax_scale * log2 e); warp-shuffle max/sum; exp2 on MUFU.
//       PV : lanes own output channels; V dequantized to fp16 like K;
//            acc += p(fp16) * v(fp16) with the same mixed-precision FMA.
//   warp 9 (epilogue): at a unit boundary inside the CTA's range each
//     consumer warp stores its raw (m, l, acc) in shared memory and arrives
//     on a hand-off mbarrier, then goes on streaming; the epilogue warp merges
//     the 8 warp states, writes the unit's output or publishes the partial,
//     takes the ticket and merges the unit if it completes it. The CTA's last
//     segment is finished by all consumer warps together.
//
// The grid is launched with programmatic dependent launch: every thread runs
// griddepcontrol.wait before the first global-memory access, so only the
// launch and the prologue overlap the previous kernel on the stream.
//
// Every mbarrier wait is bounded (kMaxPolls); on expiry the kernel records
// kDevWaitTimeout in the workspace error word, stops issuing copies, drains
// the copies it has in flight (again bounded) and returns.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <mutex>
#include <type_traits>

#include "lik_device.cuh"
#include "lik_internal.h"

namespace lik {

constexpr int kNCW = 8;                    // consumer warps
constexpr int kProducerWarp = kNCW;      // issues the bulk copies
constexpr int kEpilogueWarp = kNCW + 1;  // finishes unit segments off the streaming path
constexpr int kThreads = (kNCW + 2) * 32;
constexpr float kLog2e = 1.4426950408889634f;

template <int FMT>
struct Fmt;
template <>
struct Fmt<kF16> {
    static constexpr int ROWB = 256, T = 128, PVC = 4;
    static constexpr bool TOKK = false, TOKV = false, ZV = false, KG = false, ZK = false, SIGNED = true;
};
template <>
struct Fmt<kI8> {
    static constexpr int ROWB = 128, T = 256, PVC = 4;
    static constexpr bool TOKK = true, TOKV = true, ZV = false, KG = false, ZK = false, SIGNED = true;
};
template <>
struct Fmt<kI4Sym> {
    static constexpr int ROWB = 64, T = 256, PVC = 8;
    static constexpr bool TOKK = false, TOKV = true, ZV = false, KG = true, ZK = false, SIGNED = true;
};
template <>
struct Fmt<kI4Asym> {
    static constexpr int ROWB = 64, T = 256, PVC = 8;
    static constexpr bool TOKK = false, TOKV = true, ZV = true, KG = true, ZK = true, SIGNED = false;
};

struct DecodeParams {
    const __half* q;
    __half* out;
    const uint8_t* k;
    const uint8_t* v;
    const __half* ks;
    const __half* vs;
    const __half* kz;
    const __half* vz;
    long long seqlen, kv_buf_len, ng_buf;
    long long n_units, tpu, total_tiles;
    int n_heads, n_kv_heads, nhb;
    int group_size, tok_bulk, kg_smem, ngt;
    int n_ctas, nst, stage_bytes;
    int off_v, off_ks, off_vs, off_vz, off_kgs, off_kgz, off_q;
    int off_work, off_abuf, off_sc, off_ml, off_misc, off_bar;
    float qscale;
    // paged KV (paged != 0): caches are [num_blocks, n_kv_heads, block_size, row],
    // per-token scales [num_blocks, n_kv_heads, block_size], K group scales
    // [num_blocks, n_kv_heads, block_size / group_size, 128]; sequence b's
    // position t lives in block block_tables[b * max_blocks + t / block_size].
    const int* block_tables;
    const int* ctx_lens;
    int paged, block_size, max_blocks;
    float* part;
    unsigned* counters;
    int* err;
};

// ---- small helpers --------------------------------------------------------

template <int HB>
__device__ __forceinline__ int head_of_lane(int lane) {
    int h = 0;
#pragma unroll
    for (int L = 0, n = HB; L < 3 && n > 1; ++L, n >>= 1) h += ((lane >> L) & 1) * (n >> 1);
    return h;
}

template <int HB>
__device__ __forceinline__ int lane_of_head(int h) {
    int lane = 0;
#pragma unroll
    for (int L = 0, n = HB; L < 3 && n > 1; ++L, n >>= 1) lane |= ((h / (n >> 1)) & 1) << L, h %= (n >> 1);
    return lane;
}

// Sum v[0..HB) over the 8 lanes of a group (lane bits 0..2), scattering heads:
// afterwards the lane holds the full sum of head head_of_lane<HB>(lane).
template <int HB>
__device__ __forceinline__ float reduce_scatter8(float (&v)[HB], int lane) {
    float a[HB];
#pragma unroll
    for (int i = 0; i < HB; ++i) a[i] = v[i];
    int n = HB;
#pragma unroll
    for (int L = 0; L < 3; ++L) {
        const int m = 1 << L;
        if (n > 1) {
            const int half = n >> 1;
            const bool up = (lane >> L) & 1;
#pragma unroll
            for (int i = 0; i < HB / 2; ++i) {
                if (i < half) {
                    const float send = up ? a[i] : a[i + half];
                    const float keep = up ? a[i + half] : a[i];
                    a[i] = keep + __shfl_xor_sync(kFull, send, m);
                }
            }
            n = half;
        } else {
            a[0] += __shfl_xor_sync(kFull, a[0], m);
        }
    }
    return a[0];
}

__device__ __forceinline__ long long owner_cta(long long tile, long long total, int nctas) {
    return ((tile + 1) * nctas - 1) / total;
}
__device__ __forceinline__ long long cta_first_tile(long long c, long long total, int nctas) {
    return c * total / nctas;
}

// One step of the log-sum-exp merge of unit segments (running m, l, a) with
// segment (ms, ls, as), with explicit roundings (no contraction left to the
// compiler); a segment with ms = -inf (no positions) is an exact identity.
__device__ __forceinline__ void lse_fold(float& mg, float& lg, float& ag, float ms, float ls, float as) {
    const float mn = fmaxf(mg, ms);
    const float fa = mg == -INFINITY ? 0.f : fast_exp2(mg - mn);
    const float fb = ms == -INFINITY ? 0.f : fast_exp2(ms - mn);
    lg = fmaf(lg, fa, __fmul_rn(ls, fb));
    ag = fmaf(ag, fa, __fmul_rn(as, fb));
    mg = mn;
}
constexpr int kMergeBatch = 4;  // segments whose loads are issued together

template <int HB>
__device__ __forceinline__ float pick(const float (&x)[HB], int h) {
    float r = x[0];
#pragma unroll
    for (int hx = 1; hx < HB; ++hx)
        if (h == hx) r = x[hx];
    return r;
}

// Combine of the eight consumer warps' raw states of one unit segment, read
// from shared memory (mlb: m and l per (warp, head); abuf: 128 raw
// accumulators per (warp, head)). Lane j of the calling warp (j = lane & 7;
// lanes 8..31 repeat lanes 0..7) takes consumer warp j: the head maxima M, the
// warp weights exp2(m_j - M) and the sums L are reduced with shuffles, with
// the same result in every lane of every warp that runs it.
template <int HB>
struct WarpCombine {
    float M[HB], L[HB], fw[HB];
    __device__ __forceinline__ void load(const float* mlb, int lane) {
        const int wsrc = lane & 7;
#pragma unroll
        for (int h = 0; h < HB; ++h) {
            const float mw = mlb[(wsrc * HB + h) * 3];
            const float lw = mlb[(wsrc * HB + h) * 3 + 1];
            float mx = fmaxf(mw, __shfl_xor_sync(kFull, mw, 1));
            mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, 2));
            mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, 4));
            // a segment of a paged sequence can hold no position (M = -inf)
            const float f = mx == -INFINITY ? 0.f : fast_exp2(mw - mx);
            float ls = __fmul_rn(lw, f);
            ls += __shfl_xor_sync(kFull, ls, 1);
            ls += __shfl_xor_sync(kFull, ls, 2);
            ls += __shfl_xor_sync(kFull, ls, 4);
            M[h] = mx;
            L[h] = ls;
            fw[h] = f;
        }
    }
    // sum over the consumer warps of weight * raw accumulator of output o
    // (o >> 7 is the head; it must be the same across the calling warp)
    __device__ __forceinline__ float combined(const float* abuf, int o) const {
        const int h = o >> 7;
        const float fh = pick<HB>(fw, h);
        float x[kNCW];
#pragma unroll
        for (int ww = 0; ww < kNCW; ++ww) x[ww] = abuf[(ww * HB + h) * kHeadDim + (o & 127)];
        float a = 0.f;
#pragma unroll
        for (int ww = 0; ww < kNCW; ++ww) a = fmaf(__shfl_sync(kFull, fh, ww), x[ww], a);
        return a;
    }
};

// Hand-off of a finished unit segment from the consumer warps to the
// epilogue warp (shared memory, written by consumer warp 0 lane 0 before its
// release-arrive on the hand-off barrier).
struct EpiDesc {
    long long unit, qoff, slot;
    int whole, pad;
};

// The merge of a split unit's segments: a log-sum-exp fold, in CTA order,
// over their partials in the workspace, normalised into `out`. Threads wl,
// wl + nw, ... each produce outputs; two outputs per pass so that all their
// loads are in flight together.
// The CTAs whose ranges hold a unit: c_lo .. c_hi. CTA c_lo's segment sits
// in its second partial slot unless its range starts exactly at the unit's
// first tile (lo_first); every later CTA's segment is its first unit (slot 0).
// (64-bit divisions: computed off the end-of-kernel critical path.)
struct UnitSpan {
    long long c_lo, c_hi;
    bool lo_first;
};
__device__ __forceinline__ UnitSpan unit_span(const DecodeParams& p, long long unit) {
    UnitSpan u;
    u.c_lo = owner_cta(unit * p.tpu, p.total_tiles, p.n_ctas);
    u.c_hi = owner_cta((unit + 1) * p.tpu - 1, p.total_tiles, p.n_ctas);
    u.lo_first = cta_first_tile(u.c_lo, p.total_tiles, p.n_ctas) == unit * p.tpu;
    return u;
}

template <int HB>
__device__ __forceinline__ void merge_segments(const DecodeParams& p, const UnitSpan& sp, long long qoff, int wl,
                                               int nw) {
    constexpr int SB = kMergeBatch;
    constexpr int HBK = HB * kHeadDim;
    constexpr int SL = HBK + 2 * HB;
    const long long c_lo = sp.c_lo;
    const int nseg = static_cast<int>(sp.c_hi - c_lo + 1);
    const bool lo_first = sp.lo_first;
    for (int o0 = wl; o0 < HBK; o0 += 2 * nw) {
        float mg[2], lg[2], ag[2];
#pragma unroll
        for (int r = 0; r < 2; ++r) mg[r] = -INFINITY, lg[r] = 0.f, ag[r] = 0.f;
        for (int s0 = 0; s0 < nseg; s0 += SB) {
            float ms[2][SB], ls[2][SB], as[2][SB];
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                const int o = o0 + r * nw;
                const int h = (o < HBK ? o : 0) >> 7;
#pragma unroll
                for (int k = 0; k < SB; ++k) {
                    const long long c2 = c_lo + s0 + k;
                    const bool ok = s0 + k < nseg && o < HBK;
                    const float* q2 = p.part + (2 * (ok ? c2 : c_lo) + ((ok && c2 == c_lo && !lo_first) ? 1 : 0)) * SL;
                    ms[r][k] = ok ? __ldcg(q2 + HBK + h) : -INFINITY;
                    ls[r][k] = ok ? __ldcg(q2 + HBK + HB + h) : 0.f;
                    as[r][k] = ok ? __ldcg(q2 + o) : 0.f;
                }
            }
#pragma unroll
            for (int r = 0; r < 2; ++r)
#pragma unroll
                for (int k = 0; k < SB; ++k) lse_fold(mg[r], lg[r], ag[r], ms[r][k], ls[r][k], as[r][k]);
        }
#pragma unroll
        for (int r = 0; r < 2; ++r)
            if (o0 + r * nw < HBK) p.out[qoff + o0 + r * nw] = __float2half_rn(ag[r] / lg[r]);
    }
}

// Count this segment's partial towards its unit (acquire-release, GPU scope:
// publishes the partial written before the call and, for the last arriver,
// makes the other segments' partials visible). True when this segment
// completes the unit; the counter is then reset for the next launch.
__device__ __forceinline__ bool unit_ticket(const DecodeParams& p, long long unit, const UnitSpan& sp) {
    const unsigned old = atomic_add_acq_rel_gpu(&p.counters[unit], 1u);
    const bool last = old == static_cast<unsigned>(sp.c_hi - sp.c_lo);
    if (last) p.counters[unit] = 0u;
    return last;
}

// The HB fp16 softmax weights of one position as (HB+1)/2 packed words.
template <int HB>
__device__ __forceinline__ void load_pw(const uint16_t* src, uint32_t (&pw)[(HB + 1) / 2]) {
    if constexpr (HB == 8) {
        const uint4 u = *reinterpret_cast<const uint4*>(src);
        pw[0] = u.x; pw[1] = u.y; pw[2] = u.z; pw[3] = u.w;
    } else if constexpr (HB == 4) {
        const uint2 u = *reinterpret_cast<const uint2*>(src);
        pw[0] = u.x; pw[1] = u.y;
    } else if constexpr (HB == 2) {
        pw[0] = *reinterpret_cast<const uint32_t*>(src);
    } else {
        pw[0] = src[0];
    }
}

// acc[h][2i], acc[h][2i+1] += p_h * v[i] for every head h
template <int HB, int NV, int PVC>
__device__ __forceinline__ void pv_accum(const uint32_t (&pw)[(HB + 1) / 2], const uint32_t (&v)[NV],
                                         float (&acc)[HB][PVC]) {
#pragma unroll
    for (int h = 0; h < HB; ++h)
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            if (h & 1)
                fma_p_h2<1>(pw[h >> 1], v[i], acc[h][2 * i], acc[h][2 * i + 1]);
            else
                fma_p_h2<0>(pw[h >> 1], v[i], acc[h][2 * i], acc[h][2 * i + 1]);
        }
}

__device__ __forceinline__ float h2_sum(half2 a) {
    const float2 f = __half22float2(a);
    return f.x + f.y;
}

// ---- optional timeline probes (diagnostic builds only: -DLIK_TIMELINE) ------
#ifdef LIK_TIMELINE
__device__ unsigned long long g_lik_timeline[4096 * 12];
__device__ __forceinline__ void lik_tl(int slot) {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    g_lik_timeline[blockIdx.x * 12 + slot] = t;
    if (slot == 0) {
        unsigned sm;
        asm volatile("mov.u32 %0, %%smid;" : "=r"(sm));
        g_lik_timeline[blockIdx.x * 12 + 8] = sm;
    }
}
#define LIK_TL(cond, slot) \
    do {                   \
        if (cond) lik_tl(slot); \
    } while (0)
#else
#define LIK_TL(cond, slot) \
    do {                   \
    } while (0)
#endif

// ---- the kernel -----------------------------------------------------------

template <int FMT, int HB>
__global__ void __launch_bounds__(kThreads, 1) decode_kernel(const DecodeParams p) {
    using F = Fmt<FMT>;
    constexpr int T = F::T;
    constexpr int ROWB = F::ROWB;
    constexpr int TW = T / kNCW;  // positions per warp per tile
    constexpr int NP = TW / 4;    // QK passes (4 positions per pass)
    constexpr int PVC = F::PVC;
    constexpr int SL = HB * kHeadDim + 2 * HB;  // partial slot stride (floats)

    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    // per stage: "full" (q, K and its scales landed), "fullv" (V and its
    // scales landed) and "empty" (all consumer warps are done with the stage)
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.off_bar);
    uint64_t* fullv = full + p.nst;
    uint64_t* empty = fullv + p.nst;
    // segment hand-off to the epilogue warp: "epi_full" (the eight consumer
    // warps wrote their state) and "epi_empty" (the epilogue warp has read it)
    uint64_t* epi_full = empty + p.nst;
    uint64_t* epi_empty = epi_full + 1;
    volatile int* misc = reinterpret_cast<volatile int*>(smem + p.off_misc);
    EpiDesc* desc = reinterpret_cast<EpiDesc*>(smem + p.off_misc + 16);
    float* abuf = reinterpret_cast<float*>(smem + p.off_abuf);
    float* mlb = reinterpret_cast<float*>(smem + p.off_ml);

    const long long cta = blockIdx.x;
    const long long tb = cta_first_tile(cta, p.total_tiles, p.n_ctas);
    const long long te = cta_first_tile(cta + 1, p.total_tiles, p.n_ctas);

    if (tid == 0) {
        for (int s = 0; s < p.nst; ++s) {
            mbar_init(&full[s], 32);
            mbar_init(&fullv[s], 32);
            mbar_init(&empty[s], kNCW);
        }
        mbar_init(epi_full, kNCW);
        mbar_init(epi_empty, 1);
        misc[0] = 0;  // abort
        misc[1] = 0;  // merge ticket result
        fence_barrier_init();
    }
    // Programmatic dependent launch: this grid may start while the previous
    // kernel on the stream is still finishing; nothing in global memory is
    // read or written before that kernel has completed.
    grid_dependency_wait();
    __syncthreads();
    LIK_TL(tid == 0, 0);

    // ======================= producer warp ================================
    if (warp == kProducerWarp) {
        const uint64_t pol = l2_policy_evict_first();
        long long j = 0;
        bool ok = true;
        // incremental (stage, phase) and (unit, tile) counters: no divisions in the loop
        int st = 0;
        uint32_t ph = 0;
        long long unit = tb / p.tpu;
        long long ti = tb - unit * p.tpu;
        long long bk = unit / p.nhb;
        for (long long i = tb; i < te; ++i, ++j) {
            if (j >= p.nst) {
                const uint32_t par = ph ^ 1u;
                bool got = false;
                for (uint32_t it = 0; it < kMaxPolls; ++it) {
                    if (mbar_try_wait(&empty[st], par)) {
                        got = true;
                        break;
                    }
                    if (misc[0]) break;
                }
                if (!got) {
                    ok = false;
                    break;
                }
            }
            const long long t0 = ti * T;
            const long long seq_b = bk / p.n_kv_heads;
            const long long kvh_p = bk - seq_b * p.n_kv_heads;
            long long len_b = p.seqlen;
            if (p.paged) {
                const long long cl = p.ctx_lens[seq_b];
                len_b = cl < 0 ? 0 : (cl > p.seqlen ? p.seqlen : cl);
            }
            const int ntok = static_cast<int>(max(0LL, min(static_cast<long long>(T), len_b - t0)));
            const long long rowbase = bk * p.kv_buf_len + t0;
            uint8_t* sb = smem + static_cast<size_t>(st) * p.stage_bytes;
            const int n8 = (ntok + 7) & ~7;

            // Scales that cannot use a bulk copy (unaligned slabs): plain loads.
            if ((F::TOKK || F::TOKV) && !p.tok_bulk && !p.paged) {
                for (int t = lane; t < ntok; t += 32) {
                    if (F::TOKK) reinterpret_cast<__half*>(sb + p.off_ks)[t] = p.ks[rowbase + t];
                    if (F::TOKV) reinterpret_cast<__half*>(sb + p.off_vs)[t] = p.vs[rowbase + t];
                    if (F::ZV) reinterpret_cast<__half*>(sb + p.off_vz)[t] = p.vz[rowbase + t];
                }
            }
            const bool new_unit = (j == 0 || ti == 0);
            if (lane == 0 && p.paged) {
                // gather the tile block by block (one bulk copy per block touched)
                const int bs = p.block_size;
                const int* bt = p.block_tables + seq_b * p.max_blocks;
                uint32_t bytes_k = new_unit ? HB * kHeadDim * 2 : 0, bytes_v = 0;
                for (long long pos = t0; pos < t0 + ntok;) {
                    const int off = static_cast<int>(pos % bs);
                    const int n = static_cast<int>(min(static_cast<long long>(bs - off), t0 + ntok - pos));
                    const int nn8 = (n + 7) & ~7;
                    bytes_k += n * ROWB + (F::TOKK ? nn8 * 2 : 0);
                    bytes_v += n * ROWB + (F::TOKV ? nn8 * 2 : 0) + (F::ZV ? nn8 * 2 : 0);
                    if (F::KG && p.kg_smem)
                        bytes_k += (F::ZK ? 2 : 1) * ((pos + n - 1) / p.group_size - pos / p.group_size + 1) *
                                   kHeadDim * 2;
                    pos += n;
                }
                mbar_arrive_expect_tx(&full[st], bytes_k);
                mbar_arrive_expect_tx(&fullv[st], bytes_v);
                if (new_unit) {
                    const int hb = static_cast<int>(unit - bk * p.nhb);
                    const long long qo = (seq_b * p.n_heads + kvh_p * p.nhb * HB + hb * HB) * kHeadDim;
                    bulk_g2s(sb + p.off_q, p.q + qo, HB * kHeadDim * 2, &full[st], pol);
                }
                const long long g0 = F::KG ? t0 / p.group_size : 0;
                for (long long pos = t0; pos < t0 + ntok;) {
                    const int off = static_cast<int>(pos % bs);
                    const int n = static_cast<int>(min(static_cast<long long>(bs - off), t0 + ntok - pos));
                    const int nn8 = (n + 7) & ~7;
                    const long long page = bt[pos / bs];
                    const long long row = (page * p.n_kv_heads + kvh_p) * bs + off;
                    const int d = static_cast<int>(pos - t0);
                    bulk_g2s(sb + d * ROWB, p.k + row * ROWB, n * ROWB, &full[st], pol);
                    bulk_g2s(sb + p.off_v + d * ROWB, p.v + row * ROWB, n * ROWB, &fullv[st], pol);
                    if (F::TOKK) bulk_g2s(sb + p.off_ks + d * 2, p.ks + row, nn8 * 2, &full[st], pol);
                    if (F::TOKV) bulk_g2s(sb + p.off_vs + d * 2, p.vs + row, nn8 * 2, &fullv[st], pol);
                    if (F::ZV) bulk_g2s(sb + p.off_vz + d * 2, p.vz + row, nn8 * 2, &fullv[st], pol);
                    if (F::KG && p.kg_smem) {
                        const long long ga = pos / p.group_size, gb2 = (pos + n - 1) / p.group_size;
                        const long long gsrc = ((page * p.n_kv_heads + kvh_p) * (bs / p.group_size) +
                                                off / p.group_size) * kHeadDim;
                        const int gcnt = static_cast<int>(gb2 - ga + 1);
                        bulk_g2s(sb + p.off_kgs + (ga - g0) * kHeadDim * 2, p.ks + gsrc, gcnt * kHeadDim * 2,
                                 &full[st], pol);
                        if (F::ZK)
                            bulk_g2s(sb + p.off_kgz + (ga - g0) * kHeadDim * 2, p.kz + gsrc, gcnt * kHeadDim * 2,
                                     &full[st], pol);
                    }
                    pos += n;
                }
            } else if (lane == 0) {
                uint32_t bytes_k = ntok * ROWB + (new_unit ? HB * kHeadDim * 2 : 0);
                uint32_t bytes_v = ntok * ROWB;
                int g0 = 0, ngrp = 0;
                if ((F::TOKK || F::TOKV) && p.tok_bulk) {
                    bytes_k += F::TOKK * n8 * 2;
                    bytes_v += (F::TOKV + F::ZV) * n8 * 2;
                }
                if (F::KG && p.kg_smem && ntok > 0) {
                    g0 = static_cast<int>(t0) / p.group_size;
                    const int g1 = (static_cast<int>(t0) + ntok - 1) / p.group_size;
                    ngrp = g1 - g0 + 1;
                    bytes_k += (F::ZK ? 2 : 1) * ngrp * kHeadDim * 2;
                }
                // K side first: QK can start while V is still in flight
                mbar_arrive_expect_tx(&full[st], bytes_k);
                if (new_unit) {
                    const int hb = static_cast<int>(unit - bk * p.nhb);
                    const long long b = bk / p.n_kv_heads;
                    const long long kvh = bk - b * p.n_kv_heads;
                    const long long qo = (b * p.n_heads + kvh * p.nhb * HB + hb * HB) * kHeadDim;
                    bulk_g2s(sb + p.off_q, p.q + qo, HB * kHeadDim * 2, &full[st], pol);
                }
                bulk_g2s(sb, p.k + rowbase * ROWB, ntok * ROWB, &full[st], pol);
                if (F::TOKK && p.tok_bulk) bulk_g2s(sb + p.off_ks, p.ks + rowbase, n8 * 2, &full[st], pol);
                if (F::KG && p.kg_smem && ntok > 0) {
                    const long long gb = (bk * p.ng_buf + g0) * kHeadDim;
                    bulk_g2s(sb + p.off_kgs, p.ks + gb, ngrp * kHeadDim * 2, &full[st], pol);
                    if (F::ZK) bulk_g2s(sb + p.off_kgz, p.kz + gb, ngrp * kHeadDim * 2, &full[st], pol);
                }
                mbar_arrive_expect_tx(&fullv[st], bytes_v);
                bulk_g2s(sb + p.off_v, p.v + rowbase * ROWB, ntok * ROWB, &fullv[st], pol);
                if (p.tok_bulk) {
                    if (F::TOKV) bulk_g2s(sb + p.off_vs, p.vs + rowbase, n8 * 2, &fullv[st], pol);
                    if (F::ZV) bulk_g2s(sb + p.off_vz, p.vz + rowbase, n8 * 2, &fullv[st], pol);
                }
            } else {
                mbar_arrive(&full[st]);
                mbar_arrive(&fullv[st]);
            }
            if (++st == p.nst) {
                st = 0;
                ph ^= 1u;
            }
            if (++ti == p.tpu) {
                ti = 0;
                ++unit;
                bk = unit / p.nhb;
            }
        }
        if (!ok) {
            // Let the copies already issued land before the CTA can exit.
            const long long first = j > p.nst ? j - p.nst : 0;
            for (long long jj = first; jj < j; ++jj) {
                mbar_wait_bounded(&full[jj % p.nst], static_cast<uint32_t>((jj / p.nst) & 1));
                mbar_wait_bounded(&fullv[jj % p.nst], static_cast<uint32_t>((jj / p.nst) & 1));
            }
            if (lane == 0) atomicExch(p.err, kDevWaitTimeout);
        }
        // Every copy is issued: the next kernel on the stream may be scheduled
        // (it waits for this grid to complete before it touches memory).
        // Measured on B200 with back-to-back steps: this early trigger saves
        // about 1 us per INT8 / INT4 step and costs about 0.7 us per fp16
        // step, so fp16 leaves the trigger to the CTA's exit.
        if (FMT != kF16) grid_launch_dependents();
        return;
    }

    // ======================= epilogue warp ================================
    // Every unit segment but the CTA's last is finished here while the
    // consumer warps go on streaming: combine the eight warp states, then
    // either write the whole unit's output or publish this CTA's partial, take
    // the unit's ticket and, if this segment completes the unit, merge it.
    if (warp == kEpilogueWarp) {
        constexpr int HBK = HB * kHeadDim;
        const long long nhand = (te - 1) / p.tpu - tb / p.tpu;  // segment ends before the last
        for (long long k = 0; k < nhand; ++k) {
            if (!mbar_wait_bounded(epi_full, static_cast<uint32_t>(k & 1))) {
                misc[0] = 1;
                if (lane == 0) atomicExch(p.err, kDevWaitTimeout);
                break;
            }
            const EpiDesc d = *desc;
            WarpCombine<HB> wc;
            wc.load(mlb, lane);
            if (d.whole) {
                for (int o = lane; o < HBK; o += 32)
                    p.out[d.qoff + o] = __float2half_rn(wc.combined(abuf, o) / pick<HB>(wc.L, o >> 7));
                __syncwarp();
                if (lane == 0) mbar_arrive(epi_empty);
            } else {
                float* sp = p.part + d.slot * SL;
                for (int o = lane; o < HBK; o += 32) sp[o] = wc.combined(abuf, o);
                if (lane < HB) {
                    sp[HBK + lane] = pick<HB>(wc.M, lane);
                    sp[HBK + HB + lane] = pick<HB>(wc.L, lane);
                }
                __syncwarp();  // the partial is written; the shared state is free again
                if (lane == 0) mbar_arrive(epi_empty);
                const UnitSpan span = unit_span(p, d.unit);
                int last = 0;
                if (lane == 0) last = unit_ticket(p, d.unit, span);
                last = __shfl_sync(kFull, last, 0);
                if (last) merge_segments<HB>(p, span, d.qoff, lane, 32);
            }
        }
        return;
    }

    // ======================= consumer warps ===============================
    const int w = warp;
    const int grp = lane >> 3;
    const int jl = lane & 7;
    // QK reduce-scatter layout: QG passes of HB heads reduced together; lane
    // bits [0, log2 QG) select the pass, the next bits the head, the rest of
    // the 8-lane group holds duplicates (only when QG * HB < 8).
    constexpr int QG = (8 / HB) < NP ? (8 / HB) : NP;
    constexpr int QV = QG * HB;
    constexpr int NGRP = NP / QG;
    static_assert(NP % QG == 0, "passes must group evenly");
    constexpr int LQG = QG >= 8 ? 3 : QG >= 4 ? 2 : QG >= 2 ? 1 : 0;
    constexpr int LQV = QV >= 8 ? 3 : QV >= 4 ? 2 : QV >= 2 ? 1 : 0;
    const int qpl = head_of_lane<QG>(lane & 7);            // pass within the group
    const int hh = head_of_lane<HB>((lane & 7) >> LQG);     // head
    const bool prim = ((lane & 7) >> LQV) == 0;            // not a duplicate
    const int nct = kNCW * 32;

    uint16_t* pbuf = reinterpret_cast<uint16_t*>(smem + p.off_work) + w * TW * HB;  // p as f16
    const long long first_unit_of_cta = tb / p.tpu;
    long long nhand = 0;  // segments handed to the epilogue warp so far
    // span of the CTA's last unit, needed right after its final segment;
    // computed now, while the first tiles are still in flight, and kept in
    // shared memory (read after the final segment's barriers)
    UnitSpan* last_span = reinterpret_cast<UnitSpan*>(smem + p.off_misc + 16 + sizeof(EpiDesc));
    if (tid == 0) *last_span = unit_span(p, (te - 1) / p.tpu);

    float m_run = -INFINITY, l_run = 0.f;
    float acc[HB][PVC];
    uint32_t qh[HB][8];  // q * softmax_scale * log2e as half2, in the format's pair order
    // INT8: K codes enter the dot product as 1152 + code (fp16, exact); this
    // per-head term, -1152 * (sum of the lane's 16 q values), starts the
    // lane's partial sum and cancels the offset
    float kbias[HB];
#pragma unroll
    for (int h = 0; h < HB; ++h) kbias[h] = 0.f;
    uint32_t kg[8];      // INT4: K group scale of the lane's 16 channels (pair order)
    uint32_t kgz[8];     // INT4 asym: K group zero
    long long cur_unit = -1, seg_t0 = 0, qoff = 0, bk = 0, seq_len = 0;
    int cur_g = -1;
    int gnext = 0;  // INT4: first position (within the unit) of the next K group
    bool aborted = false;
#pragma unroll
    for (int c = 0; c < 8; ++c) kg[c] = kgz[c] = 0u;

    int st = 0;
    uint32_t ph = 0;
    long long unit = tb / p.tpu;
    long long ti = tb - unit * p.tpu;
    for (long long i = tb; i < te; ++i) {
        const bool new_unit = (unit != cur_unit);
        if (new_unit) {
            // ---- start of a unit segment ----
            cur_unit = unit;
            seg_t0 = ti;
            cur_g = -1;
            bk = unit / p.nhb;
            const int hb = static_cast<int>(unit - bk * p.nhb);
            const long long b = bk / p.n_kv_heads;
            const int kvh = static_cast<int>(bk - b * p.n_kv_heads);
            qoff = (b * p.n_heads + static_cast<long long>(kvh) * p.nhb * HB + hb * HB) * kHeadDim;
            seq_len = p.seqlen;
            if (p.paged) {
                const long long cl = p.ctx_lens[b];
                seq_len = cl < 0 ? 0 : (cl > p.seqlen ? p.seqlen : cl);
            }
            m_run = -INFINITY;
            l_run = 0.f;
#pragma unroll
            for (int h = 0; h < HB; ++h)
#pragma unroll
                for (int c = 0; c < PVC; ++c) acc[h][c] = 0.f;
        }

        if (!aborted) {
            if (misc[0] || !mbar_wait_bounded(&full[st], ph)) {
                aborted = true;
                misc[0] = 1;
                if (lane == 0) atomicExch(p.err, kDevWaitTimeout);
            }
        }
        LIK_TL(tid == 0 && new_unit && i != tb, 11);
        if (new_unit) {
            // q for the HB heads arrived with this stage (the producer copies it
            // into the first stage of every unit segment)
            const __half* sq = reinterpret_cast<const __half*>(smem + static_cast<size_t>(st) * p.stage_bytes + p.off_q);
#pragma unroll
            for (int h = 0; h < HB; ++h) {
                const __half* qp = sq + h * kHeadDim;
                // the lane's 16 QK channels, as 16 halves in channel order
                uint4 ua, ub;
                if (FMT == kF16) {
                    ua = *reinterpret_cast<const uint4*>(qp + 8 * jl);
                    ub = *reinterpret_cast<const uint4*>(qp + 64 + 8 * jl);
                } else {
                    ua = *reinterpret_cast<const uint4*>(qp + 16 * jl);
                    ub = *reinterpret_cast<const uint4*>(qp + 16 * jl + 8);
                }
                const __half* ha = reinterpret_cast<const __half*>(&ua);
                const __half* hbv = reinterpret_cast<const __half*>(&ub);
                float qf[16];
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    qf[c] = __half2float(ha[c]) * p.qscale;
                    qf[8 + c] = __half2float(hbv[c]) * p.qscale;
                }
                if (F::KG) {
                    // pair (wd*4 + k) = channels (8wd + k, 8wd + k + 4) of the lane's 16
#pragma unroll
                    for (int wd = 0; wd < 2; ++wd)
#pragma unroll
                        for (int k = 0; k < 4; ++k)
                            qh[h][wd * 4 + k] = as_u32(__floats2half2_rn(qf[8 * wd + k], qf[8 * wd + k + 4]));
                } else {
#pragma unroll
                    for (int c = 0; c < 8; ++c) qh[h][c] = as_u32(__floats2half2_rn(qf[2 * c], qf[2 * c + 1]));
                }
                if (FMT == kI8) {
                    float lo = 0.f, hi = 0.f;
                    const uint32_t off = 0x64806480u;  // (1152, 1152)
#pragma unroll
                    for (int c = 0; c < 8; ++c) fma_h2_2acc(qh[h][c], off, lo, hi);
                    kbias[h] = -(lo + hi);
                }
            }
        }
        LIK_TL(tid == 0 && i == tb, 1);

        const long long t0 = ti * T;
        const int ntok = static_cast<int>(max(0LL, min(static_cast<long long>(T), seq_len - t0)));
        const uint8_t* sb = smem + static_cast<size_t>(st) * p.stage_bytes;
        const int wt0 = w * TW;

        if (!aborted && wt0 < ntok) {
            const uint8_t* sK = sb;
            const uint8_t* sV = sb + p.off_v;
            const __half* sks = reinterpret_cast<const __half*>(sb + p.off_ks);
            const __half* svs = reinterpret_cast<const __half*>(sb + p.off_vs);
            const __half* svz = reinterpret_cast<const __half*>(sb + p.off_vz);
            const int nval = min(TW, ntok - wt0);

            // ---------------- QK ----------------
            // K is dequantized to fp16 with the oracle's rounding (fp16(code *
            // scale [+ zero])); products f16 x f16 are exact, sums in fp32.
            // Passes (4 positions each) are processed QG at a time so that,
            // after the 8-lane reduce-scatter of QG*HB partial sums, every lane
            // holds exactly one distinct (position, head) score.
            // K group scale (and zero) of group g for the lane's 16 channels
            auto load_group = [&](int g) {
                cur_g = g;
                gnext = (g + 1) * p.group_size;
                const __half* gsp;
                const __half* gzp = nullptr;
                if (p.kg_smem) {
                    const int g0 = static_cast<int>(t0) / p.group_size;
                    gsp = reinterpret_cast<const __half*>(sb + p.off_kgs) + (g - g0) * kHeadDim;
                    if (F::ZK) gzp = reinterpret_cast<const __half*>(sb + p.off_kgz) + (g - g0) * kHeadDim;
                } else {
                    long long gb = (bk * p.ng_buf + g) * kHeadDim;
                    if (p.paged) {
                        const long long pos = static_cast<long long>(g) * p.group_size;
                        const long long sq = bk / p.n_kv_heads;
                        const long long page = p.block_tables[sq * p.max_blocks + pos / p.block_size];
                        gb = ((page * p.n_kv_heads + (bk - sq * p.n_kv_heads)) *
                                  (p.block_size / p.group_size) + (pos % p.block_size) / p.group_size) *
                             kHeadDim;
                    }
                    gsp = p.ks + gb;
                    if (F::ZK) gzp = p.kz + gb;
                }
                const uint4 s0 = *reinterpret_cast<const uint4*>(gsp + 16 * jl);
                const uint4 s1 = *reinterpret_cast<const uint4*>(gsp + 16 * jl + 8);
                const __half* sh0 = reinterpret_cast<const __half*>(&s0);
                const __half* sh1 = reinterpret_cast<const __half*>(&s1);
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    kg[k] = as_u32(__halves2half2(sh0[k], sh0[k + 4]));
                    kg[4 + k] = as_u32(__halves2half2(sh1[k], sh1[k + 4]));
                }
                if (F::ZK) {
                    const uint4 z0 = *reinterpret_cast<const uint4*>(gzp + 16 * jl);
                    const uint4 z1 = *reinterpret_cast<const uint4*>(gzp + 16 * jl + 8);
                    const __half* zh0 = reinterpret_cast<const __half*>(&z0);
                    const __half* zh1 = reinterpret_cast<const __half*>(&z1);
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        kgz[k] = as_u32(__halves2half2(zh0[k], zh0[k + 4]));
                        kgz[4 + k] = as_u32(__halves2half2(zh1[k], zh1[k + 4]));
                    }
                }
            };
            // When the warp's positions of this tile lie in one K group (group
            // sizes that are multiples of 32), its scales are loaded once here
            // and the unrolled passes carry no reload code.
            bool group_checks = false;
            if constexpr (F::KG) {
                const int pos_lo = static_cast<int>(t0) + wt0;
                const int g_lo = pos_lo / p.group_size;
                if (g_lo == (pos_lo + nval - 1) / p.group_size) {
                    if (g_lo != cur_g) load_group(g_lo);
                } else {
                    group_checks = true;
                }
            }
            float sc[NGRP];
            // INT4: the groups of passes run as a rolled loop (a shorter hot
            // loop) and park their scores in the warp's shared-memory slots
            float* scs = reinterpret_cast<float*>(smem + p.off_sc) + w * NGRP * 32;
            auto qk_tile = [&](auto check_tag) {
            constexpr bool CHECK = decltype(check_tag)::value;
#pragma unroll(F::KG ? 1 : 16)
            for (int gq = 0; gq < NGRP; ++gq) {
                float vals[QV];
#pragma unroll
                for (int pl2 = 0; pl2 < QG; ++pl2) {
                    const int tt = wt0 + (gq * QG + pl2) * 4 + grp;
                    float part[HB], part2[HB];
#pragma unroll
                    for (int h = 0; h < HB; ++h) {
                        part[h] = FMT == kI8 ? kbias[h] : 0.f;
                        part2[h] = 0.f;
                    }
                    if (tt < ntok) {
                        const uint8_t* row = sK + tt * ROWB;
                        uint32_t kk[8];
                        if (FMT == kF16) {
                            const uint4 ka = *reinterpret_cast<const uint4*>(row + jl * 16);
                            const uint4 kb = *reinterpret_cast<const uint4*>(row + 128 + jl * 16);
                            kk[0] = ka.x; kk[1] = ka.y; kk[2] = ka.z; kk[3] = ka.w;
                            kk[4] = kb.x; kk[5] = kb.y; kk[6] = kb.z; kk[7] = kb.w;
                        } else if (FMT == kI8) {
                            // codes as 1152 + code (offset cancelled by kbias); the
                            // token scale multiplies the reduced score
                            const uint4 ka = *reinterpret_cast<const uint4*>(row + jl * 16);
                            i8x4_to_h2_offset(ka.x, kk[0], kk[1]);
                            i8x4_to_h2_offset(ka.y, kk[2], kk[3]);
                            i8x4_to_h2_offset(ka.z, kk[4], kk[5]);
                            i8x4_to_h2_offset(ka.w, kk[6], kk[7]);
                        } else {
                            const int tabs = static_cast<int>(t0) + tt;
                            if (CHECK && (cur_g < 0 || tabs >= gnext)) load_group(tabs / p.group_size);
                            const uint2 kw = *reinterpret_cast<const uint2*>(row + jl * 8);
                            half2 c0[4], c1[4];
                            i4x8_to_h2<F::SIGNED>(kw.x, c0);
                            i4x8_to_h2<F::SIGNED>(kw.y, c1);
    #pragma unroll
                            for (int k = 0; k < 4; ++k) {
                                if (F::ZK) {
                                    kk[k] = as_u32(__hfma2(c0[k], as_h2(kg[k]), as_h2(kgz[k])));
                                    kk[4 + k] = as_u32(__hfma2(c1[k], as_h2(kg[4 + k]), as_h2(kgz[4 + k])));
                                } else {
                                    kk[k] = as_u32(__hmul2(c0[k], as_h2(kg[k])));
                                    kk[4 + k] = as_u32(__hmul2(c1[k], as_h2(kg[4 + k])));
                                }
                            }
                        }
#pragma unroll
                        for (int c = 0; c < 8; ++c)
#pragma unroll
                            for (int h = 0; h < HB; ++h) fma_h2_2acc(qh[h][c], kk[c], part[h], part2[h]);
                    }
#pragma unroll
                    for (int h = 0; h < HB; ++h) vals[pl2 * HB + h] = part[h] + part2[h];
                }
                float s = reduce_scatter8<QV>(vals, lane);
                const int tt = wt0 + (gq * QG + qpl) * 4 + grp;
                if (tt >= ntok) {
                    s = -INFINITY;
                } else if (F::TOKK) {
                    s *= __half2float(sks[tt]);
                }
                if constexpr (F::KG)
                    scs[gq * 32 + lane] = s;
                else
                    sc[gq] = s;
            }
            if constexpr (F::KG) {
#pragma unroll
                for (int gq = 0; gq < NGRP; ++gq) sc[gq] = scs[gq * 32 + lane];
            }
            };
            if (group_checks)
                qk_tile(std::true_type{});
            else
                qk_tile(std::false_type{});

            // ---------------- online softmax (log2 domain) ----------------
            // lanes sharing a head differ in the pass bits (xor 1 .. QG/2) and
            // the position-group bits (xor 8, 16)
            float mloc = sc[0];
#pragma unroll
            for (int gq = 1; gq < NGRP; ++gq) mloc = fmaxf(mloc, sc[gq]);
#pragma unroll
            for (int m = 1; m < QG; m <<= 1) mloc = fmaxf(mloc, __shfl_xor_sync(kFull, mloc, m));
            mloc = fmaxf(mloc, __shfl_xor_sync(kFull, mloc, 8));
            mloc = fmaxf(mloc, __shfl_xor_sync(kFull, mloc, 16));
            const float mnew = fmaxf(m_run, mloc);
            const float alpha = fast_exp2(m_run - mnew);
            float ls = 0.f;
#pragma unroll
            for (int gq = 0; gq < NGRP; ++gq) {
                const int tl = (gq * QG + qpl) * 4 + grp;  // position within the warp's share
                const float e = fast_exp2(sc[gq] - mnew);
                ls += e;
                if (tl < nval && prim) pbuf[tl * HB + hh] = __half_as_ushort(__float2half_rn(e));
            }
#pragma unroll
            for (int m = 1; m < QG; m <<= 1) ls += __shfl_xor_sync(kFull, ls, m);
            ls += __shfl_xor_sync(kFull, ls, 8);
            ls += __shfl_xor_sync(kFull, ls, 16);
            l_run = fmaf(l_run, alpha, ls);
            m_run = mnew;
            float al[HB];
#pragma unroll
            for (int h = 0; h < HB; ++h) al[h] = __shfl_sync(kFull, alpha, lane_of_head<HB>(h) * QG);
            __syncwarp();
#pragma unroll
            for (int h = 0; h < HB; ++h)
#pragma unroll
                for (int c = 0; c < PVC; ++c) acc[h][c] *= al[h];

            // ---------------- PV ----------------
            if (misc[0] || !mbar_wait_bounded(&fullv[st], ph)) {
                aborted = true;
                misc[0] = 1;
                if (lane == 0) atomicExch(p.err, kDevWaitTimeout);
            }
            // V dequantized to fp16 as the oracle does; acc += p(f16) * v(f16) in fp32.
            if (FMT == kF16 || FMT == kI8) {
                // per-tile base pointers; the full-tile loop is unrolled so
                // every per-position offset is an immediate
                const uint8_t* vrow = sV + wt0 * ROWB + lane * (FMT == kF16 ? 8 : 4);
                const __half* vsr = svs + wt0;
                auto pv_token = [&](int t) {
                    uint32_t v0, v1;
                    if (FMT == kF16) {
                        const uint2 vv = *reinterpret_cast<const uint2*>(vrow + t * ROWB);
                        v0 = vv.x;
                        v1 = vv.y;
                    } else {
                        const uint32_t vv = *reinterpret_cast<const uint32_t*>(vrow + t * ROWB);
                        half2 lo, hi;
                        i8x4_to_h2(vv, lo, hi);
                        const half2 s2 = __half2half2(vsr[t]);
                        v0 = as_u32(__hmul2(lo, s2));
                        v1 = as_u32(__hmul2(hi, s2));
                    }
                    uint32_t pw[(HB + 1) / 2];
                    load_pw<HB>(pbuf + t * HB, pw);
                    const uint32_t vv2[2] = {v0, v1};
                    pv_accum<HB, 2, PVC>(pw, vv2, acc);
                };
                if (nval == TW) {
                    constexpr int U = TW <= 16 ? TW : 8;
#pragma unroll 1
                    for (int t0u = 0; t0u < TW; t0u += U) {
#pragma unroll
                        for (int t = 0; t < U; ++t) pv_token(t0u + t);
                    }
                } else {
                    for (int t = 0; t < nval; ++t) pv_token(t);
                }
            } else {
                const int hw = lane >> 4;
                const int l16 = lane & 15;
                const uint8_t* vrow = sV + (wt0 + hw) * ROWB + l16 * 4;
                const __half* vsr = svs + wt0 + hw;
                const __half* vzr = svz + wt0 + hw;
                const uint16_t* prow = pbuf + hw * HB;
                // u = position offset relative to this half-warp's first position
                auto pv_token = [&](int u) {
                    const uint32_t vv = *reinterpret_cast<const uint32_t*>(vrow + u * ROWB);
                    half2 o[4];
                    i4x8_to_h2<F::SIGNED>(vv, o);
                    const half2 s2 = __half2half2(vsr[u]);
                    uint32_t vd[4];
                    if (F::ZV) {
                        const half2 z2 = __half2half2(vzr[u]);
#pragma unroll
                        for (int k = 0; k < 4; ++k) vd[k] = as_u32(__hfma2(o[k], s2, z2));
                    } else {
#pragma unroll
                        for (int k = 0; k < 4; ++k) vd[k] = as_u32(__hmul2(o[k], s2));
                    }
                    uint32_t pw[(HB + 1) / 2];
                    load_pw<HB>(prow + u * HB, pw);
                    pv_accum<HB, 4, PVC>(pw, vd, acc);
                };
                if (nval == TW) {
#pragma unroll 4
                    for (int u = 0; u < TW; u += 2) pv_token(u);
                } else {
                    for (int u = 0; u + hw < nval; u += 2) pv_token(u);
                }
            }
            __syncwarp();
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);

        // ---------------- end of a unit segment ----------------
        // Each warp stores its raw state (m, l, acc) in shared memory. A
        // segment that is not the CTA's last is handed to the epilogue warp
        // and the consumers go straight on to the next tile; the last one is
        // finished here by all consumer warps together.
        if (ti == p.tpu - 1 || i == te - 1) {
            const bool final_seg = (i == te - 1);
            const bool whole = (seg_t0 == 0 && ti == p.tpu - 1);
            LIK_TL(tid == 0 && final_seg, 4);
            if (PVC == 8) {
#pragma unroll
                for (int h = 0; h < HB; ++h)
#pragma unroll
                    for (int c = 0; c < 8; ++c) acc[h][c] += __shfl_xor_sync(kFull, acc[h][c], 16);
            }
            // the epilogue warp has read the previous hand-off
            if (lane == 0 && nhand > 0 &&
                !mbar_wait_bounded(epi_empty, static_cast<uint32_t>((nhand - 1) & 1))) {
                misc[0] = 1;
                atomicExch(p.err, kDevWaitTimeout);
            }
            __syncwarp();
            if (grp == 0 && prim && qpl == 0) {
                mlb[(w * HB + hh) * 3] = m_run;
                mlb[(w * HB + hh) * 3 + 1] = l_run;
            }
#pragma unroll
            for (int h = 0; h < HB; ++h) {
                float* dst = abuf + (w * HB + h) * kHeadDim;
                if (PVC == 4) {
                    *reinterpret_cast<float4*>(dst + lane * 4) =
                        make_float4(acc[h][0], acc[h][1], acc[h][2], acc[h][3]);
                } else if (lane < 16) {
                    *reinterpret_cast<float4*>(dst + lane * 8) =
                        make_float4(acc[h][0], acc[h][2], acc[h][4], acc[h][6]);
                    *reinterpret_cast<float4*>(dst + lane * 8 + 4) =
                        make_float4(acc[h][1], acc[h][3], acc[h][5], acc[h][7]);
                }
            }
            // the segment's state now lives in shared memory; the next segment
            // starts from zero (clearing here also frees the registers)
            m_run = -INFINITY;
            l_run = 0.f;
#pragma unroll
            for (int h = 0; h < HB; ++h)
#pragma unroll
                for (int c = 0; c < PVC; ++c) acc[h][c] = 0.f;
            if (!final_seg) {
                if (w == 0 && lane == 0) {
                    EpiDesc d;
                    d.unit = unit;
                    d.qoff = qoff;
                    d.slot = 2 * cta + (unit == first_unit_of_cta ? 0 : 1);
                    d.whole = whole ? 1 : 0;
                    d.pad = 0;
                    *desc = d;
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(epi_full);  // release: the state and descriptor
                ++nhand;
            } else {
                named_bar_sync(1, nct);  // every warp's state is in shared memory
                LIK_TL(tid == 0, 5);
                WarpCombine<HB> wc;
                wc.load(mlb, lane);
                if (whole) {
                    for (int o = tid; o < HB * kHeadDim; o += nct)
                        p.out[qoff + o] = __float2half_rn(wc.combined(abuf, o) / pick<HB>(wc.L, o >> 7));
                } else {
                    const long long slot = 2 * cta + (unit == first_unit_of_cta ? 0 : 1);
                    float* sp = p.part + slot * SL;
                    for (int o = tid; o < HB * kHeadDim; o += nct) sp[o] = wc.combined(abuf, o);
                    if (tid < HB) {
                        sp[HB * kHeadDim + tid] = pick<HB>(wc.M, tid);
                        sp[HB * kHeadDim + HB + tid] = pick<HB>(wc.L, tid);
                    }
                    named_bar_sync(1, nct);  // the whole partial is written
                    if (tid == 0) misc[1] = unit_ticket(p, unit, *last_span) ? 1 : 0;
                    named_bar_sync(1, nct);
                    LIK_TL(tid == 0, 6);
                    if (misc[1]) merge_segments<HB>(p, *last_span, qoff, tid, nct);
                }
            }
        }
        if (++st == p.nst) {
            st = 0;
            ph ^= 1u;
        }
        if (++ti == p.tpu) {
            ti = 0;
            ++unit;
        }
        LIK_TL(tid == 0 && i == te - 2, 2);
    }
    LIK_TL(tid == 0, 3);
}

// ---- host side ------------------------------------------------------------

int heads_per_unit(int64_t group, int fmt) {
    // Eight heads per unit need more registers than the INT8/INT4 paths have
    // (168 per thread at 10 warps per SM); those formats split a group of 8
    // into two units of 4.
    if (group % 8 == 0 && fmt == kF16) return 8;
    if (group % 4 == 0) return 4;
    if (group % 2 == 0) return 2;
    return 1;
}

// Workspace layout (bytes): [error word | partial slots | unit counters].
// The partial-slot region has a fixed capacity (two slots per SM at the
// largest slot stride), so the counters always start at the same offset:
// calls with different shapes sharing one workspace never find a counter on
// top of another call's partial results. Counters are left zero by every call.
static size_t partial_region_bytes(int sm_count) {
    return align_up(static_cast<size_t>(2) * sm_count * (8 * kHeadDim + 2 * 8) * 4, 256);
}

size_t decode_workspace_bytes(int64_t batch, int64_t n_heads, int64_t n_kv_heads, int sm_count) {
    if (batch <= 0 || n_kv_heads <= 0 || n_heads <= 0) return kWsErrBytes;
    const int64_t n_units = batch * n_heads;  // upper bound over every heads-per-unit choice
    return kWsErrBytes + partial_region_bytes(sm_count) + align_up(static_cast<size_t>(n_units) * 4, 256);
}

namespace {

template <int FMT, int HB>
lik_status launch_t(const DecodeArgs& a, const DeviceInfo& di, cudaStream_t stream, std::string& err) {
    using F = Fmt<FMT>;
    constexpr int T = F::T;
    DecodeParams p{};
    p.q = static_cast<const __half*>(a.q);
    p.out = static_cast<__half*>(a.out);
    p.k = static_cast<const uint8_t*>(a.k);
    p.v = static_cast<const uint8_t*>(a.v);
    p.ks = static_cast<const __half*>(a.k_scale);
    p.vs = static_cast<const __half*>(a.v_scale);
    p.kz = static_cast<const __half*>(a.k_zero);
    p.vz = static_cast<const __half*>(a.v_zero);
    p.seqlen = a.seqlen;
    p.kv_buf_len = a.kv_buf_len;
    p.ng_buf = a.n_groups_buf;
    p.n_heads = static_cast<int>(a.n_heads);
    p.n_kv_heads = static_cast<int>(a.n_kv_heads);
    const int64_t g = a.n_heads / a.n_kv_heads;
    p.nhb = static_cast<int>(g / HB);
    p.n_units = a.batch * a.n_kv_heads * p.nhb;
    p.tpu = (a.seqlen + T - 1) / T;
    p.total_tiles = p.n_units * p.tpu;
    p.group_size = static_cast<int>(F::KG ? a.group_size : 1);
    p.paged = a.block_tables != nullptr ? 1 : 0;
    p.block_tables = a.block_tables;
    p.ctx_lens = a.context_lens;
    p.block_size = static_cast<int>(a.block_size);
    p.max_blocks = static_cast<int>(a.max_blocks);
    p.qscale = a.softmax_scale * kLog2e;

    // Per-token scales ride the bulk copy when every tile's scale run is
    // 16-byte aligned and a multiple of 16 bytes (rounded up to 8 tokens,
    // which stays inside the slab because kv_buf_len % 8 == 0).
    auto al16 = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; };
    bool tok_bulk = (a.kv_buf_len % 8 == 0);
    if (F::TOKK) tok_bulk = tok_bulk && al16(a.k_scale);
    if (F::TOKV) tok_bulk = tok_bulk && al16(a.v_scale);
    if (F::ZV) tok_bulk = tok_bulk && al16(a.v_zero);
    p.tok_bulk = tok_bulk ? 1 : 0;
    bool kg_smem = F::KG && a.group_size >= 32 && al16(a.k_scale) && (!F::ZK || al16(a.k_zero));
    if (p.paged) {
        p.tok_bulk = 1;  // block_size % 16 == 0 and 16-byte aligned scales (checked by the caller)
        kg_smem = kg_smem && (a.block_size % a.group_size == 0);
    }
    p.kg_smem = kg_smem ? 1 : 0;
    p.ngt = kg_smem ? static_cast<int>(std::min<int64_t>(a.n_groups_buf, (T + a.group_size - 1) / a.group_size + 1)) : 0;

    // stage layout
    int off = 2 * T * F::ROWB;
    p.off_v = T * F::ROWB;
    p.off_ks = off;
    if (F::TOKK) off += T * 2;
    p.off_vs = off;
    if (F::TOKV) off += T * 2;
    p.off_vz = off;
    if (F::ZV) off += T * 2;
    p.off_kgs = off;
    off += p.ngt * kHeadDim * 2;
    p.off_kgz = off;
    if (F::ZK) off += p.ngt * kHeadDim * 2;
    off = static_cast<int>(align_up(off, 16));
    p.off_q = off;
    off += HB * kHeadDim * 2;
    p.stage_bytes = static_cast<int>(align_up(off, 128));

    // per-warp fp16 softmax weights, then the per-warp raw accumulators
    const int pbuf_bytes = static_cast<int>(align_up(static_cast<size_t>(kNCW) * (T / kNCW) * HB * 2, 16));
    const int abuf_bytes = kNCW * HB * kHeadDim * 4;
    // INT4 formats: per-warp score slots (one float per lane and pass group)
    constexpr int kNP = T / kNCW / 4;
    constexpr int kQG = (8 / HB) < kNP ? (8 / HB) : kNP;
    const int sc_bytes = F::KG ? kNCW * (kNP / kQG) * 32 * 4 : 0;
    const int work = pbuf_bytes + abuf_bytes + sc_bytes;
    const int fixed = work + kNCW * HB * 3 * 4 + 80 + (3 * 8 + 2) * 8;
    int nst = (di.max_smem_optin - fixed - 256) / p.stage_bytes;
    nst = std::min(nst, 8);
    if (nst < 2) {
        err = "shared memory too small for two pipeline stages";
        return LIK_ERR_UNSUPPORTED;
    }
    // Never more stages than one CTA can use.
    p.nst = nst;
    size_t o2 = static_cast<size_t>(nst) * p.stage_bytes;
    p.off_work = static_cast<int>(o2);
    p.off_abuf = static_cast<int>(o2 + pbuf_bytes);
    p.off_sc = static_cast<int>(o2 + pbuf_bytes + abuf_bytes);
    o2 += work;
    p.off_ml = static_cast<int>(o2);
    o2 += kNCW * HB * 3 * 4;
    o2 = align_up(o2, 16);
    p.off_misc = static_cast<int>(o2);
    o2 += 16 + sizeof(EpiDesc) + sizeof(UnitSpan);
    o2 = align_up(o2, 8);
    p.off_bar = static_cast<int>(o2);
    o2 += (3 * nst + 2) * 8;
    const size_t smem = o2;

    p.n_ctas = static_cast<int>(std::min<long long>(p.total_tiles, di.sm_count));

    uint8_t* ws = static_cast<uint8_t*>(a.workspace);
    p.err = reinterpret_cast<int*>(ws);
    p.part = reinterpret_cast<float*>(ws + kWsErrBytes);
    p.counters = reinterpret_cast<unsigned*>(ws + kWsErrBytes + partial_region_bytes(di.sm_count));
    const size_t need = kWsErrBytes + partial_region_bytes(di.sm_count) +
                        align_up(static_cast<size_t>(p.n_units) * 4, 256);
    if (a.workspace == nullptr || a.workspace_bytes < need) {
        err = "workspace too small: need " + std::to_string(need) + " bytes";
        return LIK_ERR_WORKSPACE;
    }

    auto kern = decode_kernel<FMT, HB>;
    static std::once_flag once[64];
    static cudaError_t attr_err[64];
    int dev = 0;
    cudaGetDevice(&dev);
    const int slot = dev & 63;
    std::call_once(once[slot], [&] {
        attr_err[slot] = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, di.max_smem_optin);
    });
    if (attr_err[slot] != cudaSuccess) {
        err = std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(attr_err[slot]);
        return LIK_ERR_CUDA;
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(p.n_ctas);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, p);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) {
        err = std::string("decode kernel launch: ") + cudaGetErrorString(e);
        return LIK_ERR_CUDA;
    }
    return LIK_OK;
}

template <int FMT>
lik_status launch_fmt(const DecodeArgs& a, const DeviceInfo& di, cudaStream_t s, std::string& err) {
    switch (heads_per_unit(a.n_heads / a.n_kv_heads, FMT)) {
        case 8:
            if constexpr (FMT == kF16) return launch_t<FMT, 8>(a, di, s, err);
            err = "internal: eight heads per unit is fp16-only";
            return LIK_ERR_UNSUPPORTED;
        case 4: return launch_t<FMT, 4>(a, di, s, err);
        case 2: return launch_t<FMT, 2>(a, di, s, err);
        default: return launch_t<FMT, 1>(a, di, s, err);
    }
}

}  // namespace

lik_status launch_decode(const DecodeArgs& a, cudaStream_t stream, std::string& err) {
    DeviceInfo di;
    if (!device_info(di, err)) return LIK_ERR_CUDA;
    switch (a.fmt) {
        case kF16: return launch_fmt<kF16>(a, di, stream, err);
        case kI8: return launch_fmt<kI8>(a, di, stream, err);
        case kI4Sym: return launch_fmt<kI4Sym>(a, di, stream, err);
        case kI4Asym: return launch_fmt<kI4Asym>(a, di, stream, err);
        default: err = "unknown KV format"; return LIK_ERR_INVALID_ARGUMENT;
    }
}

}  // namespace lik
