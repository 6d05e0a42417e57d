// Single-query GQA decode attention over an fp16 / INT8-per-token / INT4-KIVI
// KV cache for sm_100a, with the dequantization fused into a split-sequence
// (FlashDecoding) loop and the log-sum-exp combine fused into the same launch.
//
// Work decomposition
//   unit  = (batch, kv_head, head block): HB query heads that share one KV
//           slab (HB = the GQA group, or a divisor of it), so every KV byte is
//           read from HBM exactly once per step (the reference launches one
//           CTA per query head and re-reads each slab G times, relying on L2).
//   tile  = T consecutive KV positions of one unit (fp16 128, INT8 / INT4
//           256 positions: 32-64 KB of codes).
//   The flattened (unit, tile) sequence is split evenly over a persistent grid
//   of one CTA per SM: CTA c owns tiles [c*TT/C, (c+1)*TT/C). A CTA's range may
//   cover whole units (written straight to `out`) and partial units at its
//   two ends (written as an un-normalised partial to the workspace; the CTA
//   that completes a unit's last partial, found with an atomic ticket, merges
//   them). No CTA ever waits for another CTA.
//
// Inside a CTA
//   warp 8 (producer): lane 0 posts each stage's transaction bytes, then the
//     lanes issue the tile's 1-D bulk async copies together (cp.async.bulk,
//     no tensor map, no multicast): K and V rows, q with a unit's first tile,
//     per-token / per-group scales and zeros, into an NST-deep shared-memory
//     ring. Each stage has a "full" (q, K) and a "fullv" (V) mbarrier with
//     transaction bytes and an "empty" mbarrier the consumers arrive on.
//   warps 0-7 (consumers, tensor pipe): each warp owns 16-position m-tiles
//     of the tiles and keeps its own online-softmax state (m, l, acc) for the
//     HB heads. Per m-tile:
//       QK : mma.sync with K rows as A and the heads as the 8 columns of B.
//            fp16: f16 m16n8k16 on q. INT8 / INT4: integer m16n8k32 on the
//            raw codes (INT4 nibbles by masking) against q folded with the
//            scales as byte limbs of 16 / 24-bit fixed point; the limbs are
//            combined in fp32 (exact).
//       softmax: log2 domain; the running maximum is raised only when a
//            score exceeds it by more than kTau (one warp vote per tile).
//       PV : f16 m16n8k16 with V^T as A and p^T (from the QK accumulator by
//            movmatrix.trans) as B; INT8 / INT4 V codes enter as fp16
//            subnormals with p * v_scale as the weight.
//     INT4 folds the tile's K group scales into q first (one slice per warp,
//     then a named barrier); with four heads per unit the consumers form two
//     groups of four warps that take tiles in turn. Other INT4 group sizes
//     (not multiples of 16) use a CUDA-core consumer that dequantizes to fp16
//     exactly as the reference oracle does and multiplies with
//     fma.rn.f32.f16.
//   warp 9 (epilogue): at a unit boundary inside the CTA's range each
//     consumer warp stores its raw (m, l, acc) in shared memory and arrives
//     on a hand-off mbarrier, then goes on streaming; the epilogue warp merges
//     the 8 warp states, writes the unit's output or publishes the partial,
//     takes the ticket and merges the unit if it completes it. The CTA's last
//     segment is finished by all consumer warps together.
//
// The grid is launched with programmatic dependent launch: every thread runs
// griddepcontrol.wait before its first global-memory access, so only the
// launch, the prologue and the producer's first address arithmetic overlap
// the previous kernel on the stream.
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
template <int FMT, bool MMA>
constexpr int threads_for() {
    return kThreads;
}
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

// Division by a launch constant with one multiply-high (dividends and
// divisors below 2^31; the host rejects launches beyond that):
// q = (umulhi(x, m) + x) >> s with s = ceil(log2 d), m = 2^32 (2^s - d) / d + 1.
// Keeps 64-bit integer division (an inlined ~80-instruction sequence per
// site) out of the streaming loops.
struct FDiv {
    uint32_t d, m, s;
    __device__ __forceinline__ long long q(long long x) const {
        const uint32_t xx = static_cast<uint32_t>(x);
        return static_cast<long long>((__umulhi(xx, m) + xx) >> s);
    }
    __device__ __forceinline__ long long r(long long x) const { return x - q(x) * static_cast<long long>(d); }
};

inline FDiv make_fdiv(uint32_t d) {
    FDiv f{d, 0u, 0u};
    while ((uint64_t{1} << f.s) < d) ++f.s;
    f.m = static_cast<uint32_t>(((uint64_t{1} << 32) * ((uint64_t{1} << f.s) - d)) / d + 1);
    return f;
}

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
    int off_w, off_zk, ngw;  // tensor-pipe INT4 path: per-stage folded K weights, group constants, groups
    float qscale;
    // paged KV (paged != 0): caches are [num_blocks, n_kv_heads, block_size, row],
    // per-token scales [num_blocks, n_kv_heads, block_size], K group scales
    // [num_blocks, n_kv_heads, block_size / group_size, 128]; sequence b's
    // position t lives in block block_tables[b * max_blocks + t / block_size].
    const int* block_tables;
    const int* ctx_lens;
    long long num_blocks;  // pages in the cache; table entries outside [0, num_blocks) are rejected
    int paged, block_size, max_blocks, off_ntok;
    float* part;
    unsigned* counters;
    int* err;
    FDiv fd_tpu, fd_nhb, fd_hkv, fd_gs, fd_bs, fd_nst;
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

// A block-table entry used for a direct global read: out-of-range entries
// record kDevBadBlock and read page 0 instead (the tile they belong to is
// masked by the producer).
__device__ __forceinline__ long long checked_page(const DecodeParams& p, long long page) {
    if (page < 0 || page >= p.num_blocks) {
        atomicExch(p.err, kDevBadBlock);
        return 0;
    }
    return page;
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


// The consumer warps' side of a unit segment's end, once every warp has
// stored its raw state (m, l per head in mlb; standard accumulators in abuf).
// Not the CTA's last segment: hand it to the epilogue warp and go on
// streaming. The CTA's last segment: combine the warp states here (all
// consumer warps), then write the unit's output or publish the partial, take
// the unit's ticket and merge the unit if this segment completes it.
// The CTA's last segment, finished by all consumer warps together.
template <int HB>
__device__ __forceinline__ void finish_final_segment(const DecodeParams& p, bool whole, long long unit, long long qoff,
                                                  long long slot, volatile int* misc, const float* mlb,
                                                  const float* abuf, const UnitSpan* last_span, int lane, int tid) {
    constexpr int nct = kNCW * 32;
    named_bar_sync(1, nct);  // every warp's state is in shared memory
    WarpCombine<HB> wc;
    wc.load(mlb, lane);
    if (whole) {
        for (int o = tid; o < HB * kHeadDim; o += nct)
            p.out[qoff + o] = __float2half_rn(wc.combined(abuf, o) / pick<HB>(wc.L, o >> 7));
    } else {
        float* sp = p.part + slot * (HB * kHeadDim + 2 * HB);
        for (int o = tid; o < HB * kHeadDim; o += nct) sp[o] = wc.combined(abuf, o);
        if (tid < HB) {
            sp[HB * kHeadDim + tid] = pick<HB>(wc.M, tid);
            sp[HB * kHeadDim + HB + tid] = pick<HB>(wc.L, tid);
        }
        named_bar_sync(1, nct);  // the whole partial is written
        if (tid == 0) misc[1] = unit_ticket(p, unit, *last_span) ? 1 : 0;
        named_bar_sync(1, nct);
        if (misc[1]) merge_segments<HB>(p, *last_span, qoff, tid, nct);
    }
}

// The consumer warps' side of a unit segment's end, once every warp has
// stored its raw state (m, l per head in mlb; standard accumulators in abuf).
// Not the CTA's last segment: hand it to the epilogue warp and go on
// streaming. The CTA's last segment: combine the warp states here (all
// consumer warps), then write the unit's output or publish the partial, take
// the unit's ticket and merge the unit if this segment completes it.
template <int HB>
__device__ __forceinline__ void finish_segment(const DecodeParams& p, bool final_seg, bool whole, long long unit,
                                               long long qoff, long long slot, long long& nhand, EpiDesc* desc,
                                               uint64_t* epi_full, volatile int* misc, const float* mlb,
                                               const float* abuf, const UnitSpan* last_span, int w, int lane,
                                               int tid) {
    if (!final_seg) {
        if (w == 0 && lane == 0) {
            EpiDesc d;
            d.unit = unit;
            d.qoff = qoff;
            d.slot = slot;
            d.whole = whole ? 1 : 0;
            d.pad = 0;
            *desc = d;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(epi_full);  // release: the state and descriptor
        ++nhand;
        return;
    }
    finish_final_segment<HB>(p, whole, unit, qoff, slot, misc, mlb, abuf, last_span, lane, tid);
}

// One segment hand-off processed by the epilogue warp.
template <int HB>
__device__ __forceinline__ void epilogue_handoff(const DecodeParams& p, const EpiDesc& d, const float* mlb,
                                              const float* abuf, uint64_t* epi_empty, int lane) {
    constexpr int HBK = HB * kHeadDim;
    WarpCombine<HB> wc;
    wc.load(mlb, lane);
    if (d.whole) {
        for (int o = lane; o < HBK; o += 32)
            p.out[d.qoff + o] = __float2half_rn(wc.combined(abuf, o) / pick<HB>(wc.L, o >> 7));
        __syncwarp();
        if (lane == 0) mbar_arrive(epi_empty);
    } else {
        float* sp = p.part + d.slot * (HBK + 2 * HB);
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

// Before a consumer warp overwrites the shared hand-off state: the epilogue
// warp has read the previous hand-off (bounded wait).
__device__ __forceinline__ void wait_handoff_free(const DecodeParams& p, uint64_t* epi_empty, volatile int* misc,
                                                  long long nhand, int lane) {
    if (lane == 0 && nhand > 0 && !mbar_wait_bounded(epi_empty, static_cast<uint32_t>((nhand - 1) & 1))) {
        misc[0] = 1;
        atomicExch(p.err, kDevWaitTimeout);
    }
    __syncwarp();
}


// Reduce each of the N (a power of two <= 32) values over the 32 lanes of the
// warp with OP (sum or max), scattering them: afterwards lane l holds the
// full result for value `head` (the same for the 32 / N lanes that share the
// bits above log2(32 / N)). log2(N) halving exchanges plus log2(32 / N)
// butterfly steps: N - 1 + 5 - log2(N) shuffles instead of 5 N.
struct OpSum {
    template <typename T>
    __device__ __forceinline__ T operator()(T a, T b) const { return a + b; }
};
struct OpMax {
    __device__ __forceinline__ float operator()(float a, float b) const { return fmaxf(a, b); }
};
template <int N, typename T, typename OP>
__device__ __forceinline__ T lane_reduce_scatter(T (&v)[N], int lane, int& head, OP op) {
    int n = N, h = 0, b = 4;
#pragma unroll
    for (int step = 0; step < 5; ++step, --b) {
        if (n > 1) {
            const int half = n >> 1;
            const bool up = (lane >> b) & 1;
#pragma unroll
            for (int i = 0; i < N / 2; ++i) {
                if (i < half) {
                    const T send = up ? v[i] : v[i + half];
                    const T keep = up ? v[i + half] : v[i];
                    v[i] = op(keep, __shfl_xor_sync(kFull, send, 1 << b));
                }
            }
            if (up) h += half;
            n = half;
        } else {
            v[0] = op(v[0], __shfl_xor_sync(kFull, v[0], 1 << b));
        }
    }
    head = h;
    return v[0];
}
template <int N>
__device__ __forceinline__ constexpr int lane_of_result(int h) {
    return h * (32 / N);
}

// ---- tensor-pipe building blocks (INT8 / INT4 formats) --------------------
//
// QK and PV run as mma.sync m16n8k16 (f16 x f16 -> f32). Codes enter the
// tensor pipe as fp16 *subnormals*: a nibble or byte n masked into the low
// mantissa bits of a half is exactly n * 2^-24 (a nibble masked at bits 4..7 is
// 16 n * 2^-24), one LOP3 per two values and no conversion; the tensor pipe
// multiplies subnormal inputs exactly (checked on B200: no flush to zero).
// Scales and zeros never touch the codes: per-channel K group scales are folded
// into q (w_c = q_c * scale_c, fp16), per-token scales into the score (INT8 K)
// or into the softmax weight (p' = p * v_scale, fp16), and the zero points /
// code offsets become per-head constants added in fp32:
//   INT4 asym K : s = 2^24 * sum_c w_c n_c            + sum_c q_c z_c
//   INT4 sym  K : s = 2^24 * sum_c w_c (c_c + 8)      - 8 sum_c w_c
//   INT8      K : s = k_scale * (2^24 * sum_c w_c (c_c + 128) - 128 sum_c w_c)
//   V           : o = 2^24 * sum_t p'_t u_t + (sum_t p_t z_t  |  -off * sum_t p'_t)
// where u is the fed code (n, c + 8 or c + 128) and the offset sums use the
// fp16 weights actually fed to the MMA, so the offsets cancel exactly.
//
// Fragment maps (g = lane / 4, r = lane % 4; rho swaps bits 0 and 1 of a row
// index, which spreads the V rows one instruction reads over both halves of
// the shared-memory banks):
//   QK  A = K tile (16 positions x 16 channels): lane rows rho(g), rho(g) + 8;
//       channels: lane r's block of 32 (INT4: bytes 16r..16r+15 of a row,
//       INT8: bytes 32r..32r+31), in the order the masks extract them.
//       B = folded q (16 channels x 8 heads), lane column = head g.
//       D = scores (positions x heads): lane holds heads 2r, 2r+1.
//   PV  A = V^T (16 channels x 16 positions), B = p'^T (positions x heads),
//       obtained from the QK accumulator layout by movmatrix.trans.
//       D = output^T: lane holds channels 16g + 2mt (+1) of heads 2r, 2r+1.

__device__ __forceinline__ void mma_f16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                              uint32_t b0, uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
    uint32_t y;
    asm("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
    return y;
}

__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
    return as_u32(__floats2half2_rn(lo, hi));
}

// A consumer's wait for a stage: one poll when the stage has landed (the
// common case, no other access); otherwise bounded polling that also gives up
// as soon as another warp has flagged an abort in misc[0].
__device__ __forceinline__ bool stage_wait(uint64_t* bar, uint32_t parity, volatile int* misc) {
    if (mbar_try_wait(bar, parity)) return true;
#pragma unroll 1
    for (uint32_t i = 0; i < kMaxPolls; ++i) {
        if (misc[0]) return false;
        if (mbar_try_wait(bar, parity)) return true;
    }
    return false;
}

// rho: the row permutation of a 16-row MMA tile (swap bits 0 and 1)
__device__ __forceinline__ int rho(int i) { return (i & ~3) | ((i & 1) << 1) | ((i & 2) >> 1); }

template <int FMT>
struct MmaFmt {
    // nibble formats: codes as 4-bit fields; XOR turns two's complement into
    // offset binary (c + 8) for the symmetric format
    static constexpr bool I4 = FMT == kI4Sym || FMT == kI4Asym;
    static constexpr uint32_t X4 = FMT == kI4Sym ? 0x88888888u : 0u;
    static constexpr float VOFF = FMT == kI4Sym ? 8.f : FMT == kI8 ? 128.f : 0.f;  // V code offset
    // fixed-point limbs of the folded QK weights (INT8: 16 bits, INT4: 24 bits;
    // the INT4 weights carry the K group scale and need the wider range)
    static constexpr int L = I4 ? 3 : FMT == kI8 ? 2 : 1;
    // Softmax weights may reach 2^kTau before the running maximum is raised.
    // The fp16 weight p * v_scale stays finite for every fp16 V: v_scale is at
    // most 65504 / 127 (INT8) or 2 * 65504 / 15 (INT4), so p <= 64 resp. 4.
    // fp16 KV: p itself is fed (at most 2^8), the accumulators are fp32.
    static constexpr float kTau = FMT == kI8 ? 6.f : FMT == kF16 ? 8.f : 2.f;
    // byte offset of lane r's first K chunk and of lane g's V channels in a row
    static constexpr int KCB = I4 ? 16 : FMT == kI8 ? 32 : 16;
    static constexpr int VCB = I4 ? 8 : FMT == kI8 ? 16 : 32;
};

// two subnormal halves from the low (x & 0x000F000F) / high (x & 0x00F000F0)
// nibble of each 16-bit half of x (after the format's XOR)
template <int FMT>
__device__ __forceinline__ uint32_t nib_lo(uint32_t x) {
    return (x ^ MmaFmt<FMT>::X4) & 0x000F000Fu;
}
template <int FMT>
__device__ __forceinline__ uint32_t nib_hi(uint32_t x) {
    return (x ^ MmaFmt<FMT>::X4) & 0x00F000F0u;
}
// two subnormal halves from bytes 0 and 2 of x, two's complement -> c + 128
__device__ __forceinline__ uint32_t byte_pair(uint32_t x) { return (x ^ 0x00800080u) & 0x00FF00FFu; }

// Integer MMA m16n8k32 (s32 accumulate): A = K codes as bytes (s8 for INT8,
// u8 nibble values for INT4), B = one 8-bit limb of the folded q weights
// (the top limb signed, lower limbs unsigned).
template <bool AU, bool BU>
__device__ __forceinline__ void mma_i8_16832(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
    if constexpr (AU && BU)
        asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
            : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
    else if constexpr (AU && !BU)
        asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
            : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
    else if constexpr (!AU && BU)
        asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
            : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
    else
        asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
            : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// QK of one 16-position m-tile on the integer tensor pipe. K rows at krow
// (the lane's row rho(g); the second row is 8 rows further), the lane's
// 32-channel block r already offset. The folded weights are fixed point with
// L 8-bit limbs per head: B[l][ks][0..1] is the B fragment of limb l (0 = top)
// at k-step ks. d[l] receives sum_c code_c * limb_l(w_c).
//   INT8: the 32 code bytes of a row are the A fragments as loaded (k-step ks
//         uses words 2ks, 2ks+1: channels 32r + 8ks + 0..7).
//   INT4: word j of a row holds channels 32r + 8j + 0..7 as nibbles;
//         (w & 0x0F0F0F0F) gives the even channels and (w >> 4) & 0x0F0F0F0F
//         the odd ones as bytes (the symmetric format XORs 8 first: c + 8).
template <int FMT, int L>
__device__ __forceinline__ void qk_mtile_int(const uint8_t* krow, const uint32_t (&B)[L][4][2], int (&d)[L][4]) {
#pragma unroll
    for (int l = 0; l < L; ++l)
#pragma unroll
        for (int c = 0; c < 4; ++c) d[l][c] = 0;
    if constexpr (MmaFmt<FMT>::I4) {
        constexpr uint32_t X = FMT == kI4Sym ? 0x08080808u : 0u;
        const uint4 k0 = *reinterpret_cast<const uint4*>(krow);
        const uint4 k1 = *reinterpret_cast<const uint4*>(krow + 8 * 64);
        const uint32_t w0[4] = {k0.x, k0.y, k0.z, k0.w};
        const uint32_t w1[4] = {k1.x, k1.y, k1.z, k1.w};
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
            const uint32_t e0 = (w0[ks] ^ X) & 0x0F0F0F0Fu, e1 = (w1[ks] ^ X) & 0x0F0F0F0Fu;
            const uint32_t o0 = ((w0[ks] >> 4) ^ X) & 0x0F0F0F0Fu, o1 = ((w1[ks] >> 4) ^ X) & 0x0F0F0F0Fu;
#pragma unroll
            for (int l = 0; l < L; ++l) {
                if (l == 0)
                    mma_i8_16832<true, false>(d[l], e0, e1, o0, o1, B[l][ks][0], B[l][ks][1]);
                else
                    mma_i8_16832<true, true>(d[l], e0, e1, o0, o1, B[l][ks][0], B[l][ks][1]);
            }
        }
    } else {
        const uint4 k0a = *reinterpret_cast<const uint4*>(krow);
        const uint4 k0b = *reinterpret_cast<const uint4*>(krow + 16);
        const uint4 k1a = *reinterpret_cast<const uint4*>(krow + 8 * 128);
        const uint4 k1b = *reinterpret_cast<const uint4*>(krow + 8 * 128 + 16);
        const uint32_t w0[8] = {k0a.x, k0a.y, k0a.z, k0a.w, k0b.x, k0b.y, k0b.z, k0b.w};
        const uint32_t w1[8] = {k1a.x, k1a.y, k1a.z, k1a.w, k1b.x, k1b.y, k1b.z, k1b.w};
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
#pragma unroll
            for (int l = 0; l < L; ++l) {
                if (l == 0)
                    mma_i8_16832<false, false>(d[l], w0[2 * ks], w1[2 * ks], w0[2 * ks + 1], w1[2 * ks + 1],
                                               B[l][ks][0], B[l][ks][1]);
                else
                    mma_i8_16832<false, true>(d[l], w0[2 * ks], w1[2 * ks], w0[2 * ks + 1], w1[2 * ks + 1],
                                              B[l][ks][0], B[l][ks][1]);
            }
    }
}

// QK of one 16-position m-tile of an fp16 K tile on the f16 tensor pipe
// (fp32 accumulate: exact products). Lane r's channels are the 16-byte chunks
// r, r + 4, r + 8, r + 12 of a row (krow is offset to chunk r; the four lanes
// of a row read four different bank groups); k-step ks uses the lane's words
// 2ks, 2ks + 1 of those 64 bytes. B[ks] is the matching fragment of q (head g).
__device__ __forceinline__ void qk_mtile_f16(const uint8_t* krow, const uint32_t (&B)[8][2], float (&d)[4]) {
    uint32_t w0[16], w1[16];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint4 a = *reinterpret_cast<const uint4*>(krow + 64 * j);
        const uint4 b = *reinterpret_cast<const uint4*>(krow + 8 * 256 + 64 * j);
        w0[4 * j] = a.x, w0[4 * j + 1] = a.y, w0[4 * j + 2] = a.z, w0[4 * j + 3] = a.w;
        w1[4 * j] = b.x, w1[4 * j + 1] = b.y, w1[4 * j + 2] = b.z, w1[4 * j + 3] = b.w;
    }
    d[0] = d[1] = d[2] = d[3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) mma_f16_16816(d, w0[2 * ks], w1[2 * ks], w0[2 * ks + 1], w1[2 * ks + 1], B[ks][0], B[ks][1]);
}

// The fp16 in half `hf` (0: low, 1: high) of a packed word, as float.
__device__ __forceinline__ float half_of(uint32_t w, int hf) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(w >> (16 * hf))));
}

// Byte b of each of four 32-bit values, packed (value i -> byte i).
__device__ __forceinline__ uint32_t byte_lane(int v0, int v1, int v2, int v3, int b) {
    const uint32_t lo = __byte_perm(static_cast<uint32_t>(v0), static_cast<uint32_t>(v1), b | ((4 + b) << 4));
    const uint32_t hi = __byte_perm(static_cast<uint32_t>(v2), static_cast<uint32_t>(v3), b | ((4 + b) << 4));
    return __byte_perm(lo, hi, 0x5410);
}

// PV of one 16-position k-step: V rows A = vrow, B = A + 2, C = A + 8,
// D = A + 10 (positions rho(2r), rho(2r+1), rho(2r) + 8, rho(2r+1) + 8), the
// lane's 16 channels starting at byte vcol; (b0, b1) = p'^T fragment.
template <int FMT>
__device__ __forceinline__ void pv_kstep(const uint8_t* vrow, uint32_t b0, uint32_t b1, float (&acc)[8][4]) {
    if constexpr (MmaFmt<FMT>::I4) {
        constexpr int RB = 64;
        const uint2 A = *reinterpret_cast<const uint2*>(vrow);
        const uint2 B = *reinterpret_cast<const uint2*>(vrow + 2 * RB);
        const uint2 C = *reinterpret_cast<const uint2*>(vrow + 8 * RB);
        const uint2 D = *reinterpret_cast<const uint2*>(vrow + 10 * RB);
        const uint32_t a[2] = {A.x, A.y}, b[2] = {B.x, B.y}, c[2] = {C.x, C.y}, dd[2] = {D.x, D.y};
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const uint32_t ab[2] = {__byte_perm(a[j], b[j], 0x5410), __byte_perm(a[j], b[j], 0x7632)};
            const uint32_t cd[2] = {__byte_perm(c[j], dd[j], 0x5410), __byte_perm(c[j], dd[j], 0x7632)};
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const uint32_t xa = ab[t >> 1] >> ((t & 1) * 8);
                const uint32_t xc = cd[t >> 1] >> ((t & 1) * 8);
                mma_f16_16816(acc[4 * j + t], nib_lo<FMT>(xa), nib_hi<FMT>(xa), nib_lo<FMT>(xc), nib_hi<FMT>(xc), b0,
                              b1);
            }
        }
    } else if constexpr (FMT == kF16) {
        // fp16 V: the lane's 16 channels (32 bytes) of four rows; M rows g and
        // g + 8 of m-tile x are channels 16g + 2x and 16g + 2x + 1
        constexpr int RB = 256;
        uint32_t a[8], b[8], c[8], dd[8];
#pragma unroll
        for (int hv = 0; hv < 2; ++hv) {
            const uint4 A = *reinterpret_cast<const uint4*>(vrow + 16 * hv);
            const uint4 B = *reinterpret_cast<const uint4*>(vrow + 2 * RB + 16 * hv);
            const uint4 C = *reinterpret_cast<const uint4*>(vrow + 8 * RB + 16 * hv);
            const uint4 D = *reinterpret_cast<const uint4*>(vrow + 10 * RB + 16 * hv);
            a[4 * hv] = A.x, a[4 * hv + 1] = A.y, a[4 * hv + 2] = A.z, a[4 * hv + 3] = A.w;
            b[4 * hv] = B.x, b[4 * hv + 1] = B.y, b[4 * hv + 2] = B.z, b[4 * hv + 3] = B.w;
            c[4 * hv] = C.x, c[4 * hv + 1] = C.y, c[4 * hv + 2] = C.z, c[4 * hv + 3] = C.w;
            dd[4 * hv] = D.x, dd[4 * hv + 1] = D.y, dd[4 * hv + 2] = D.z, dd[4 * hv + 3] = D.w;
        }
#pragma unroll
        for (int x = 0; x < 8; ++x)
            mma_f16_16816(acc[x], __byte_perm(a[x], b[x], 0x5410), __byte_perm(a[x], b[x], 0x7632),
                          __byte_perm(c[x], dd[x], 0x5410), __byte_perm(c[x], dd[x], 0x7632), b0, b1);
    } else {
        constexpr int RB = 128;
        const uint4 A = *reinterpret_cast<const uint4*>(vrow);
        const uint4 B = *reinterpret_cast<const uint4*>(vrow + 2 * RB);
        const uint4 C = *reinterpret_cast<const uint4*>(vrow + 8 * RB);
        const uint4 D = *reinterpret_cast<const uint4*>(vrow + 10 * RB);
        const uint32_t a[4] = {A.x, A.y, A.z, A.w}, b[4] = {B.x, B.y, B.z, B.w};
        const uint32_t c[4] = {C.x, C.y, C.z, C.w}, dd[4] = {D.x, D.y, D.z, D.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
#pragma unroll
            for (int t = 0; t < 2; ++t) {
                const uint32_t xa = __byte_perm(a[j], b[j], t ? 0x7632 : 0x5410);
                const uint32_t xc = __byte_perm(c[j], dd[j], t ? 0x7632 : 0x5410);
                mma_f16_16816(acc[2 * j + t], byte_pair(xa), byte_pair(xa >> 8), byte_pair(xc), byte_pair(xc >> 8),
                              b0, b1);
            }
        }
    }
}

// ---- the kernel -----------------------------------------------------------

// INT4 fixed-point weight preparation for one tile (tensor-pipe path), run by
// every consumer warp on its share of the tile's (K group, head) slices:
// w_c = q_c * softmax_scale * log2 e * k_scale[group][c] for the 128 channels,
// as 24-bit fixed point (step = max |w| / (2^23 - 1)) split into three byte
// limbs laid out as QK B fragments, plus the head's score constant (asym:
// sum_c q_c z_c; sym: -8 * the fed weights' sum, cancelling the +8 code
// offset) and step.
// INT4 tensor pipe with four heads per unit: the consumer warps form
// kWarpGroups groups that take tiles in turn (each warp covering
// kWarpGroups x 32 positions of its group's tiles, 32 at a time), so that one
// group's weight preparation and barrier overlap the other groups'
// tensor-pipe work (measured: two groups -10% on a config-4-sized INT4
// launch; four groups -2% more there but +1.2 us at config 1). 1: all
// consumer warps share every tile.
template <int FMT, int HB, bool MMA>
constexpr int kWarpGroups = (MMA && Fmt<FMT>::KG && HB == 4) ? 2 : 1;

template <int FMT, int HB>
__device__ __forceinline__ void prep_int4_weights(const DecodeParams& p, const uint8_t* sb, long long t0, int ntok,
                                                  int gi0, int gstep, int lane, int pcb, int phf, int head,
                                                  const float (&qh)[4], long long unit) {
    using F = Fmt<FMT>;
    constexpr int L = MmaFmt<FMT>::L;
    constexpr float kFix = 8388607.f;  // 2^23 - 1
    const long long g0 = p.fd_gs.q(t0);
    const int ngrp = static_cast<int>(p.fd_gs.q(t0 + ntok - 1) - g0 + 1);
    uint32_t* bw = reinterpret_cast<uint32_t*>(const_cast<uint8_t*>(sb) + p.off_w);
    float* zk = reinterpret_cast<float*>(const_cast<uint8_t*>(sb) + p.off_zk);
    float* dq = zk + p.ngw * HB;
    const int r = lane >> 3, ks = (lane >> 1) & 3;
    // slices gi * HB + head for gi = gi0, gi0 + gstep, ...
#pragma unroll 1
    for (int gi = gi0; gi < ngrp; gi += gstep) {
        const __half* gsp;
        const __half* gzp = nullptr;
        if (p.kg_smem) {
            gsp = reinterpret_cast<const __half*>(sb + p.off_kgs) + gi * kHeadDim;
            if (F::ZK) gzp = reinterpret_cast<const __half*>(sb + p.off_kgz) + gi * kHeadDim;
        } else {
            const long long ga = g0 + gi;
            const long long bk = p.fd_nhb.q(unit);
            long long gb = (bk * p.ng_buf + ga) * kHeadDim;
            if (p.paged) {
                const long long pos = ga * p.group_size;
                const long long sq2 = p.fd_hkv.q(bk);
                const long long page = checked_page(p, p.block_tables[sq2 * p.max_blocks + p.fd_bs.q(pos)]);
                gb = ((page * p.n_kv_heads + (bk - sq2 * p.n_kv_heads)) * p.fd_gs.q(p.block_size) +
                      p.fd_gs.q(p.fd_bs.r(pos))) * kHeadDim;
            }
            gsp = p.ks + gb;
            if (F::ZK) gzp = p.kz + gb;
        }
        float wv[4], amax = 0.f, zp = 0.f;
        {
            const uint4 u = *reinterpret_cast<const uint4*>(gsp + pcb);
            const uint32_t uw[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
            for (int i2 = 0; i2 < 4; ++i2) {
                wv[i2] = qh[i2] * half_of(uw[i2], phf);
                amax = fmaxf(amax, fabsf(wv[i2]));
            }
            if (F::ZK) {
                const uint4 uz = *reinterpret_cast<const uint4*>(gzp + pcb);
                const uint32_t zw[4] = {uz.x, uz.y, uz.z, uz.w};
#pragma unroll
                for (int i2 = 0; i2 < 4; ++i2) zp = fmaf(qh[i2], half_of(zw[i2], phf), zp);
            }
        }
        // one warp reduction instruction: non-negative floats order like their bits
        amax = __uint_as_float(__reduce_max_sync(kFull, __float_as_uint(amax)));
        const float inv = amax > 0.f ? __fdividef(kFix, amax) : 0.f;
        const float step = amax > 0.f ? __fdividef(amax, kFix) : 0.f;
        int wi[4];
#pragma unroll
        for (int i2 = 0; i2 < 4; ++i2)  // clamp: w * inv can round up to 2^23 at the maximum
            wi[i2] = max(-8388607, min(8388607, __float2int_rn(wv[i2] * inv)));
        uint32_t* dst = bw + ((gi * HB + head) * 4 + r) * (L * 8) + 2 * ks + phf;
#pragma unroll
        for (int l = 0; l < L; ++l) dst[8 * l] = byte_lane(wi[0], wi[1], wi[2], wi[3], L - 1 - l);
        if (F::ZK) {
#pragma unroll
            for (int m = 1; m < 32; m <<= 1) zp += __shfl_xor_sync(kFull, zp, m);
        } else {
            const int is = __reduce_add_sync(kFull, (wi[0] + wi[1]) + (wi[2] + wi[3]));
            zp = -8.f * step * static_cast<float>(is);
        }
        if (lane == 0) {
            zk[gi * HB + head] = zp;
            dq[gi * HB + head] = step;
        }
    }
}

template <int FMT, int HB, bool MMA>
__global__ void __launch_bounds__(threads_for<FMT, MMA>(), 1) decode_kernel(const DecodeParams p) {
    using F = Fmt<FMT>;
    constexpr int T = F::T;
    constexpr int ROWB = F::ROWB;
    constexpr int TW = T / kNCW;  // positions per warp per tile
    constexpr int NP = TW / 4;    // QK passes (4 positions per pass)
    constexpr int PVC = F::PVC;

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
            mbar_init(&full[s], 1);
            mbar_init(&fullv[s], 1);
            mbar_init(&empty[s], kNCW / kWarpGroups<FMT, HB, MMA>);
        }
        mbar_init(epi_full, kNCW);
        mbar_init(epi_empty, 1);

        misc[0] = 0;  // abort
        misc[1] = 0;  // merge ticket result
        fence_barrier_init();
    }
    // Programmatic dependent launch: this grid may start while the previous
    // kernel on the stream is still finishing; nothing in global memory is
    // read or written before that kernel has completed. The producer of a
    // contiguous cache runs its first tile's address arithmetic first and
    // waits right before its first global access.
    __syncthreads();
    if (warp != kProducerWarp || p.paged) grid_dependency_wait();

    // ======================= producer warp ================================
    if (warp == kProducerWarp) {
        const uint64_t pol = l2_policy_evict_first();
        long long j = 0;
        bool ok = true;
        // incremental (stage, phase) and (unit, tile) counters: no divisions in the loop
        int st = 0;
        uint32_t ph = 0;
        long long unit = p.fd_tpu.q(tb);
        long long ti = tb - unit * p.tpu;
        long long bk = p.fd_nhb.q(unit);
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
            const long long seq_b = p.fd_hkv.q(bk);
            const long long kvh_p = bk - seq_b * p.n_kv_heads;
            long long len_b = p.seqlen;
            if (p.paged) {
                const long long cl = p.ctx_lens[seq_b];
                len_b = cl < 0 ? 0 : (cl > p.seqlen ? p.seqlen : cl);
            }
            int ntok = static_cast<int>(max(0LL, min(static_cast<long long>(T), len_b - t0)));
            const long long rowbase = bk * p.kv_buf_len + t0;
            uint8_t* sb = smem + static_cast<size_t>(st) * p.stage_bytes;
            if (p.paged) {
                // Every page the tile touches must lie inside the cache; a tile
                // with an out-of-range table entry copies nothing, records
                // kDevBadBlock and is masked (the consumers read its live
                // length from the stage).
                bool bad = false;
                if (ntok > 0) {
                    const int* bt = p.block_tables + seq_b * p.max_blocks;
                    const long long b0 = p.fd_bs.q(t0), b1 = p.fd_bs.q(t0 + ntok - 1);
                    for (long long blk = b0 + lane; blk <= b1; blk += 32) {
                        const long long page = bt[blk];
                        bad |= page < 0 || page >= p.num_blocks;
                    }
                }
                if (__any_sync(kFull, bad)) {
                    ntok = 0;
                    if (lane == 0) atomicExch(p.err, kDevBadBlock);
                }
                if (lane == 0) *reinterpret_cast<int*>(sb + p.off_ntok) = ntok;
            }
            const int n8 = (ntok + 7) & ~7;

            if (j == 0 && !p.paged) grid_dependency_wait();
            // Scales that cannot use a bulk copy (unaligned slabs): plain loads.
            if ((F::TOKK || F::TOKV) && !p.tok_bulk && !p.paged) {
                for (int t = lane; t < ntok; t += 32) {
                    if (F::TOKK) reinterpret_cast<__half*>(sb + p.off_ks)[t] = p.ks[rowbase + t];
                    if (F::TOKV) reinterpret_cast<__half*>(sb + p.off_vs)[t] = p.vs[rowbase + t];
                    if (F::ZV) reinterpret_cast<__half*>(sb + p.off_vz)[t] = p.vz[rowbase + t];
                }
                // lane 0's release-arrive below publishes the other lanes' writes
                __syncwarp();
            }
            if constexpr (FMT == kF16 && MMA) {
                // fp16 V rows past the live length up to the next 16-position
                // m-tile are fed to the PV MMA with p = 0: zero them, since
                // 0 * (stale non-finite fp16) would not vanish
                const int z1 = min((ntok + 15) & ~15, T);
                for (int idx = lane; idx < (z1 - ntok) * (ROWB / 16); idx += 32)
                    *reinterpret_cast<uint4*>(sb + p.off_v + ntok * ROWB + idx * 16) = make_uint4(0u, 0u, 0u, 0u);
                __syncwarp();
            }
            // q rides with a unit's first tile in this CTA (with its first
            // kWarpGroups tiles when consumer warp groups take tiles in turn)
            const bool new_unit = j < kWarpGroups<FMT, HB, MMA> || ti < kWarpGroups<FMT, HB, MMA>;
            if (lane == 0 && p.paged) {
                // gather the tile block by block (one bulk copy per block touched)
                const int bs = p.block_size;
                const int* bt = p.block_tables + seq_b * p.max_blocks;
                uint32_t bytes_k = new_unit ? HB * kHeadDim * 2 : 0, bytes_v = 0;
                for (long long pos = t0; pos < t0 + ntok;) {
                    const int off = static_cast<int>(p.fd_bs.r(pos));
                    const int n = static_cast<int>(min(static_cast<long long>(bs - off), t0 + ntok - pos));
                    const int nn8 = (n + 7) & ~7;
                    bytes_k += n * ROWB + (F::TOKK ? nn8 * 2 : 0);
                    bytes_v += n * ROWB + (F::TOKV ? nn8 * 2 : 0) + (F::ZV ? nn8 * 2 : 0);
                    if (F::KG && p.kg_smem)
                        bytes_k += (F::ZK ? 2 : 1) * (p.fd_gs.q(pos + n - 1) - p.fd_gs.q(pos) + 1) *
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
                const long long g0 = F::KG ? p.fd_gs.q(t0) : 0;
                for (long long pos = t0; pos < t0 + ntok;) {
                    const int off = static_cast<int>(p.fd_bs.r(pos));
                    const int n = static_cast<int>(min(static_cast<long long>(bs - off), t0 + ntok - pos));
                    const int nn8 = (n + 7) & ~7;
                    const long long page = bt[p.fd_bs.q(pos)];
                    const long long row = (page * p.n_kv_heads + kvh_p) * bs + off;
                    const int d = static_cast<int>(pos - t0);
                    bulk_g2s(sb + d * ROWB, p.k + row * ROWB, n * ROWB, &full[st], pol);
                    bulk_g2s(sb + p.off_v + d * ROWB, p.v + row * ROWB, n * ROWB, &fullv[st], pol);
                    if (F::TOKK) bulk_g2s(sb + p.off_ks + d * 2, p.ks + row, nn8 * 2, &full[st], pol);
                    if (F::TOKV) bulk_g2s(sb + p.off_vs + d * 2, p.vs + row, nn8 * 2, &fullv[st], pol);
                    if (F::ZV) bulk_g2s(sb + p.off_vz + d * 2, p.vz + row, nn8 * 2, &fullv[st], pol);
                    if (F::KG && p.kg_smem) {
                        const long long ga = p.fd_gs.q(pos), gb2 = p.fd_gs.q(pos + n - 1);
                        const long long gsrc = ((page * p.n_kv_heads + kvh_p) * p.fd_gs.q(bs) +
                                                p.fd_gs.q(off)) * kHeadDim;
                        const int gcnt = static_cast<int>(gb2 - ga + 1);
                        bulk_g2s(sb + p.off_kgs + (ga - g0) * kHeadDim * 2, p.ks + gsrc, gcnt * kHeadDim * 2,
                                 &full[st], pol);
                        if (F::ZK)
                            bulk_g2s(sb + p.off_kgz + (ga - g0) * kHeadDim * 2, p.kz + gsrc, gcnt * kHeadDim * 2,
                                     &full[st], pol);
                    }
                    pos += n;
                }
            } else if (!p.paged) {
                // One bulk copy costs the issuing thread ~200 cycles, so the
                // tile's copies are issued by different lanes in parallel,
                // after lane 0 has posted both barriers' transaction bytes.
                uint32_t bytes_k = ntok * ROWB + (new_unit ? HB * kHeadDim * 2 : 0);
                uint32_t bytes_v = ntok * ROWB;
                int g0 = 0, ngrp = 0;
                if ((F::TOKK || F::TOKV) && p.tok_bulk) {
                    bytes_k += F::TOKK * n8 * 2;
                    bytes_v += (F::TOKV + F::ZV) * n8 * 2;
                }
                if (F::KG && p.kg_smem && ntok > 0) {
                    g0 = static_cast<int>(p.fd_gs.q(t0));
                    const int g1 = static_cast<int>(p.fd_gs.q(t0 + ntok - 1));
                    ngrp = g1 - g0 + 1;
                    bytes_k += (F::ZK ? 2 : 1) * ngrp * kHeadDim * 2;
                }
                // one arrival per barrier (lane 0): per-lane arrivals are
                // serialized shared-memory atomics
                if (lane == 0) {
                    mbar_arrive_expect_tx(&full[st], bytes_k);
                    mbar_arrive_expect_tx(&fullv[st], bytes_v);
                }
                __syncwarp();
                // each lane selects one of the tile's copies; one warp-wide
                // instruction issues them all
                const void* src = nullptr;
                uint32_t dst_off = 0, nbytes = 0;
                uint64_t* bar = &full[st];
                if (lane == 0 && ntok > 0) {
                    src = p.k + rowbase * ROWB, dst_off = 0, nbytes = ntok * ROWB;
                } else if (lane == 1 && ntok > 0) {
                    src = p.v + rowbase * ROWB, dst_off = p.off_v, nbytes = ntok * ROWB, bar = &fullv[st];
                } else if (lane == 2 && new_unit) {
                    const int hb = static_cast<int>(unit - bk * p.nhb);
                    const long long b = p.fd_hkv.q(bk);
                    const long long kvh = bk - b * p.n_kv_heads;
                    src = p.q + (b * p.n_heads + kvh * p.nhb * HB + hb * HB) * kHeadDim;
                    dst_off = p.off_q, nbytes = HB * kHeadDim * 2;
                } else if (F::TOKK && lane == 3 && p.tok_bulk && ntok > 0) {
                    src = p.ks + rowbase, dst_off = p.off_ks, nbytes = n8 * 2;
                } else if (F::KG && lane == 4 && p.kg_smem && ntok > 0) {
                    src = p.ks + (bk * p.ng_buf + g0) * kHeadDim, dst_off = p.off_kgs, nbytes = ngrp * kHeadDim * 2;
                } else if (F::ZK && lane == 5 && p.kg_smem && ntok > 0) {
                    src = p.kz + (bk * p.ng_buf + g0) * kHeadDim, dst_off = p.off_kgz, nbytes = ngrp * kHeadDim * 2;
                } else if (F::TOKV && lane == 6 && p.tok_bulk && ntok > 0) {
                    src = p.vs + rowbase, dst_off = p.off_vs, nbytes = n8 * 2, bar = &fullv[st];
                } else if (F::ZV && lane == 7 && p.tok_bulk && ntok > 0) {
                    src = p.vz + rowbase, dst_off = p.off_vz, nbytes = n8 * 2, bar = &fullv[st];
                }
                if (nbytes > 0) bulk_g2s(sb + dst_off, src, nbytes, bar, pol);
            }
            if (++st == p.nst) {
                st = 0;
                ph ^= 1u;
            }
            if (++ti == p.tpu) {
                ti = 0;
                ++unit;
                bk = p.fd_nhb.q(unit);
            }
        }
        if (!ok) {
            // Let the copies already issued land before the CTA can exit.
            const long long first = j > p.nst ? j - p.nst : 0;
            for (long long jj = first; jj < j; ++jj) {
                mbar_wait_bounded(&full[p.fd_nst.r(jj)], static_cast<uint32_t>(p.fd_nst.q(jj) & 1));
                mbar_wait_bounded(&fullv[p.fd_nst.r(jj)], static_cast<uint32_t>(p.fd_nst.q(jj) & 1));
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
        const long long nhand = p.fd_tpu.q(te - 1) - p.fd_tpu.q(tb);  // segment ends before the last
        for (long long k = 0; k < nhand; ++k) {
            if (!mbar_wait_bounded(epi_full, static_cast<uint32_t>(k & 1))) {
                misc[0] = 1;
                if (lane == 0) atomicExch(p.err, kDevWaitTimeout);
                break;
            }
            const EpiDesc d = *desc;
            epilogue_handoff<HB>(p, d, mlb, abuf, epi_empty, lane);
        }
        return;
    }

    // ======================= consumer warps (tensor pipe) =================
    // Each warp takes TW / 16 consecutive 16-position m-tiles at a time and
    // runs them side by side in one straight block: the QK MMAs of all of them,
    // one softmax update (a single vote), then the PV MMAs of all of them, so
    // the independent chains overlap and the tile loop carries little control
    // flow. (With warp groups, a warp covers NG such parts of its group's
    // tiles.)
    if constexpr (MMA) {
        using M = MmaFmt<FMT>;
        const int w = warp;
        const int g = lane >> 2, r = lane & 3;
        const int rg = rho(g);
        const int vr = rho(2 * r);
        constexpr int MT = TW / 16;         // m-tiles per warp per tile
        constexpr int L = M::L;
        // output scale of the PV accumulators: 2^24 for codes fed as subnormals
        // (INT4 odd channels were fed as 16 n), 1 for fp16 V
        constexpr float kSub = FMT == kF16 ? 1.f : 16777216.f;
        constexpr float kScHi = M::I4 ? kSub / 16.f : kSub;
        constexpr int NG = kWarpGroups<FMT, HB, MMA>;
        constexpr bool SPLIT = NG > 1;
        constexpr int GW = kNCW / NG;       // warps per group
        constexpr int NHALF = NG;           // TW-position parts of a warp's share per tile
        constexpr int HPW = SPLIT ? HB / GW : 1;  // INT4: heads whose weights a warp prepares
        const int wg = w % GW;              // warp within its group
        const int wgrp = w / GW;
        const int wt0 = wg * NHALF * TW;
        // INT4: a warp's TW positions of a tile lie in one K group
        const bool one_group = F::KG && p.group_size % TW == 0;
        const long long first_unit_of_cta = p.fd_tpu.q(tb);
        long long nhand = 0;
        UnitSpan* last_span = reinterpret_cast<UnitSpan*>(smem + p.off_misc + 16 + sizeof(EpiDesc));
        if (tid == 0) *last_span = unit_span(p, p.fd_tpu.q(te - 1));

        float acc[8][4];
        float m_run[2], l_run[2], zv[2], lf[2];
        uint32_t Bq[L][4][2];  // fixed-point limbs of the folded QK weights (B fragments)
        uint32_t Bh[8][2];     // fp16 KV: q of head g as B fragments (8 k-steps)
        float zk[2], dk[2];    // per-head score constant and fixed-point step of the weights loaded
        bool aborted = false;
        auto reset_state = [&]() {
#pragma unroll
            for (int mt = 0; mt < 8; ++mt)
#pragma unroll
                for (int c = 0; c < 4; ++c) acc[mt][c] = 0.f;
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) m_run[hh] = -INFINITY, l_run[hh] = 0.f, zv[hh] = 0.f, lf[hh] = 0.f;
        };
        reset_state();
#pragma unroll
        for (int l = 0; l < L; ++l)
#pragma unroll
            for (int k2 = 0; k2 < 4; ++k2) Bq[l][k2][0] = Bq[l][k2][1] = 0u;
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) Bh[ks][0] = Bh[ks][1] = 0u;
        zk[0] = zk[1] = dk[0] = dk[1] = 0.f;
        auto fail = [&]() {
            aborted = true;
            misc[0] = 1;
            if (lane == 0) atomicExch(p.err, kDevWaitTimeout);
        };
        // INT4: the tile's fixed-point weights are prepared by all consumer warps
        // together, one (K group, head) slice per warp and pass; warp w always
        // takes head w % HB, whose q over the lane's 4 channels it keeps here
        // (lane: block lane / 8, k-step (lane / 2) % 4, half lane % 2 -> channels
        // pcb + phf + 2 i)
        const int phf = lane & 1;
        const int pcb = 32 * (lane >> 3) + 8 * ((lane >> 1) & 3);
        const int ph_head = SPLIT ? wg * HPW : w % HB;  // first of the warp's HPW heads
        // INT4: the heads of the lane's two score columns (absent heads -> head 0)
        [[maybe_unused]] const int zh0 = 2 * r < HB ? 2 * r : 0, zh1 = 2 * r + 1 < HB ? 2 * r + 1 : 0;
        float qh[HPW][4] = {};
        long long q_unit = -1;  // unit whose q is in qh

        int st = 0;
        uint32_t ph = 0;
        long long unit = p.fd_tpu.q(tb), ti = tb - unit * p.tpu, cur_unit = -1, seq_len = 0;
        for (long long i = tb; i < te; ++i) {
            const bool new_unit = unit != cur_unit;
            if (new_unit) {
                cur_unit = unit;
                seq_len = p.seqlen;
                if (p.paged) {
                    const long long cl = p.ctx_lens[p.fd_hkv.q(p.fd_nhb.q(unit))];
                    seq_len = cl < 0 ? 0 : (cl > p.seqlen ? p.seqlen : cl);
                }
            }
            // tiles alternate between the two warp groups (SPLIT); the stage and
            // segment bookkeeping below runs for every tile
            if (!SPLIT || (((i - tb) % NG) == wgrp)) {
            if (!aborted && !stage_wait(&full[st], ph, misc)) fail();
            const uint8_t* sb = smem + static_cast<size_t>(st) * p.stage_bytes;
            const long long t0 = ti * T;
            int ntok = static_cast<int>(max(0LL, min(static_cast<long long>(T), seq_len - t0)));
            if (p.paged) ntok = *reinterpret_cast<const volatile int*>(sb + p.off_ntok);
            if constexpr (FMT == kF16) {
                if (new_unit) {
                    // q of head g as given (the softmax scale is applied to the
                    // fp32 scores), lane r's chunks r + 4j of the row
                    const __half* qp = reinterpret_cast<const __half*>(sb + p.off_q) + (g < HB ? g : 0) * kHeadDim;
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        uint4 u = *reinterpret_cast<const uint4*>(qp + 8 * (r + 4 * j));
                        if (g >= HB) u = make_uint4(0u, 0u, 0u, 0u);
                        Bh[2 * j][0] = u.x, Bh[2 * j][1] = u.y, Bh[2 * j + 1][0] = u.z, Bh[2 * j + 1][1] = u.w;
                    }
                }
            }
            if constexpr (FMT == kI8) {
                if (new_unit) {
                    // q * softmax_scale * log2 e for head g over the lane block's
                    // 32 channels as 16-bit fixed point (two limbs); the step is
                    // the head's max |w| / 32767
                    const __half* qp =
                        reinterpret_cast<const __half*>(sb + p.off_q) + (g < HB ? g : 0) * kHeadDim + 32 * r;
                    float wv[32];
                    float mxw = 0.f;
#pragma unroll
                    for (int c4 = 0; c4 < 4; ++c4) {
                        const uint4 u = *reinterpret_cast<const uint4*>(qp + 8 * c4);
                        const uint32_t uw[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
                        for (int i2 = 0; i2 < 8; ++i2) {
                            wv[8 * c4 + i2] = g < HB ? half_of(uw[i2 >> 1], i2 & 1) * p.qscale : 0.f;
                            mxw = fmaxf(mxw, fabsf(wv[8 * c4 + i2]));
                        }
                    }
                    mxw = fmaxf(mxw, __shfl_xor_sync(kFull, mxw, 1));
                    mxw = fmaxf(mxw, __shfl_xor_sync(kFull, mxw, 2));
                    const float inv = mxw > 0.f ? 32767.f / mxw : 0.f;
#pragma unroll
                    for (int k2 = 0; k2 < 4; ++k2)
#pragma unroll
                        for (int hf = 0; hf < 2; ++hf) {
                            const int c0 = 8 * k2 + 4 * hf;
                            int iv[4];
#pragma unroll
                            for (int e = 0; e < 4; ++e) iv[e] = max(-32767, min(32767, __float2int_rn(wv[c0 + e] * inv)));
                            Bq[0][k2][hf] = byte_lane(iv[0], iv[1], iv[2], iv[3], 1);
                            Bq[1][k2][hf] = byte_lane(iv[0], iv[1], iv[2], iv[3], 0);
                        }
                    const float step = mxw > 0.f ? mxw / 32767.f : 0.f;
                    dk[0] = __shfl_sync(kFull, step, 8 * r);
                    dk[1] = __shfl_sync(kFull, step, 8 * r + 4);
                }
            }
            if constexpr (F::KG) {
                if (unit != q_unit) {
                    q_unit = unit;
                    // q of this warp's head arrived with the unit's first stage
                    // (of this warp group)
#pragma unroll
                    for (int hh = 0; hh < HPW; ++hh) {
                        const uint4 u = *reinterpret_cast<const uint4*>(
                            reinterpret_cast<const __half*>(sb + p.off_q) + (ph_head + hh) * kHeadDim + pcb);
                        const uint32_t uw[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
                        for (int i2 = 0; i2 < 4; ++i2) qh[hh][i2] = half_of(uw[i2], phf) * p.qscale;
                    }
                }
                if (!aborted && ntok > 0) {
#pragma unroll
                    for (int hh = 0; hh < HPW; ++hh)
                        prep_int4_weights<FMT, HB>(p, sb, t0, ntok, SPLIT ? 0 : w / HB, SPLIT ? 1 : kNCW / HB,
                                                   lane, pcb, phf, ph_head + hh, qh[hh], unit);
                }
                // every consumer warp of the tile passes here once, aborted or not
                named_bar_sync(2 + wgrp, GW * 32);
            }
            int wt = wt0;  // first position of the half in progress
            int nval = 0;
            [[maybe_unused]] int cur_gi = -1;  // INT4: K group whose weights are in Bq (this tile)
            // The common case, every position of the warp's share live, runs a
            // copy of the tile body without the per-row masking.
            auto tile_body = [&](auto full_tag) {
                constexpr bool FULL = decltype(full_tag)::value;
                [[maybe_unused]] int d[MT][L][4];  // raw QK accumulators per m-tile and limb
                [[maybe_unused]] float df[MT][4];  // fp16 KV: the QK accumulators
                float zc[MT][2], dqc[MT][2];
                if (FULL || nval > 0) {
                    // ---------------- QK (integer tensor pipe) ----------------
#pragma unroll
                    for (int mi = 0; mi < MT; ++mi) {
                        if (FULL || 16 * mi < nval) {
                            if constexpr (F::KG) {
                              if (mi == 0 || !one_group) {
                                const int gi = static_cast<int>(p.fd_gs.q(t0 + wt + 16 * mi) - p.fd_gs.q(t0));
                                if (gi != cur_gi) {
                                    cur_gi = gi;
                                    const uint4* bw = reinterpret_cast<const uint4*>(
                                        sb + p.off_w + ((gi * HB + (g < HB ? g : 0)) * 4 + r) * (L * 32));
                                    // columns of absent heads (g >= HB) repeat head 0,
                                    // weights and constants alike; their results
                                    // are never stored
#pragma unroll
                                    for (int l = 0; l < L; ++l) {
                                        const uint4 u0 = bw[2 * l], u1 = bw[2 * l + 1];
                                        Bq[l][0][0] = u0.x, Bq[l][0][1] = u0.y;
                                        Bq[l][1][0] = u0.z, Bq[l][1][1] = u0.w;
                                        Bq[l][2][0] = u1.x, Bq[l][2][1] = u1.y;
                                        Bq[l][3][0] = u1.z, Bq[l][3][1] = u1.w;
                                    }
                                    const float* zkp = reinterpret_cast<const float*>(sb + p.off_zk) + gi * HB;
                                    const float* dqp = zkp + p.ngw * HB;
                                    zk[0] = zkp[zh0];
                                    zk[1] = zkp[zh1];
                                    dk[0] = dqp[zh0];
                                    dk[1] = dqp[zh1];
                                }
                              }
                            }
                            if constexpr (FMT == kF16)
                                qk_mtile_f16(sb + (wt + 16 * mi + rg) * ROWB + M::KCB * r, Bh, df[mi]);
                            else
                                qk_mtile_int<FMT, L>(sb + (wt + 16 * mi + rg) * ROWB + M::KCB * r, Bq, d[mi]);
                            zc[mi][0] = zk[0], zc[mi][1] = zk[1];
                            dqc[mi][0] = dk[0], dqc[mi][1] = dk[1];
                        }
                    }
                }
                // every warp waits for the stage's V copies before releasing it, also
                // when none of its positions is live
                if (!aborted && !stage_wait(&fullv[st], ph, misc)) fail();
                if ((FULL || nval > 0) && !aborted) {
                    {
                        // ---------------- scores ----------------
                        float sc[MT][4];
#pragma unroll
                        for (int mi = 0; mi < MT; ++mi) {
                            [[maybe_unused]] const int row = wt + 16 * mi + rg;
                            const bool ok0 = FULL || 16 * mi + rg < nval, ok1 = FULL || 16 * mi + rg + 8 < nval;
                            float dv[4];
#pragma unroll
                            for (int c = 0; c < 4; ++c) {
                                if constexpr (FMT == kF16)
                                    dv[c] = df[mi][c];
                                else if constexpr (L == 2)
                                    dv[c] = static_cast<float>(d[mi][0][c] * 256 + d[mi][1][c]);
                                else
                                    dv[c] = fmaf(static_cast<float>(d[mi][0][c] * 256 + d[mi][1][c]), 256.f,
                                                 static_cast<float>(d[mi][2][c]));
                            }
                            if constexpr (FMT == kF16) {
#pragma unroll
                                for (int c = 0; c < 4; ++c) sc[mi][c] = dv[c] * p.qscale;
                            } else if constexpr (FMT == kI8) {
                                const __half* sks = reinterpret_cast<const __half*>(sb + p.off_ks);
                                const float k0 = __half2float(sks[row]), k1 = __half2float(sks[row + 8]);
                                sc[mi][0] = dv[0] * dqc[mi][0] * k0;
                                sc[mi][1] = dv[1] * dqc[mi][1] * k0;
                                sc[mi][2] = dv[2] * dqc[mi][0] * k1;
                                sc[mi][3] = dv[3] * dqc[mi][1] * k1;
                            } else {
                                sc[mi][0] = fmaf(dv[0], dqc[mi][0], zc[mi][0]);
                                sc[mi][1] = fmaf(dv[1], dqc[mi][1], zc[mi][1]);
                                sc[mi][2] = fmaf(dv[2], dqc[mi][0], zc[mi][0]);
                                sc[mi][3] = fmaf(dv[3], dqc[mi][1], zc[mi][1]);
                            }
                            // rows past the live length (and m-tiles past it) are masked
                            if (!ok0) sc[mi][0] = sc[mi][1] = -INFINITY;
                            if (!ok1) sc[mi][2] = sc[mi][3] = -INFINITY;
                        }
                        // ---------------- online softmax (log2 domain) ----------------
                        // The running maximum is only raised when a score exceeds it
                        // by more than kTau (weights up to 2^kTau, which keeps
                        // p * v_scale inside fp16 for every fp16 V): one vote.
                        float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
                        for (int mi = 0; mi < MT; ++mi) {
                            mx0 = fmaxf(mx0, fmaxf(sc[mi][0], sc[mi][2]));
                            mx1 = fmaxf(mx1, fmaxf(sc[mi][1], sc[mi][3]));
                        }
                        if (__any_sync(kFull, mx0 > m_run[0] + M::kTau || mx1 > m_run[1] + M::kTau)) {
                            mx0 = fmaxf(mx0, __shfl_xor_sync(kFull, mx0, 4));
                            mx1 = fmaxf(mx1, __shfl_xor_sync(kFull, mx1, 4));
                            mx0 = fmaxf(mx0, __shfl_xor_sync(kFull, mx0, 8));
                            mx1 = fmaxf(mx1, __shfl_xor_sync(kFull, mx1, 8));
                            mx0 = fmaxf(mx0, __shfl_xor_sync(kFull, mx0, 16));
                            mx1 = fmaxf(mx1, __shfl_xor_sync(kFull, mx1, 16));
                            const float mn0 = fmaxf(m_run[0], mx0), mn1 = fmaxf(m_run[1], mx1);
                            const float a0 = mn0 == -INFINITY ? 1.f : fast_exp2(m_run[0] - mn0);
                            const float a1 = mn1 == -INFINITY ? 1.f : fast_exp2(m_run[1] - mn1);
                            m_run[0] = mn0;
                            m_run[1] = mn1;
                            l_run[0] *= a0, zv[0] *= a0, lf[0] *= a0;
                            l_run[1] *= a1, zv[1] *= a1, lf[1] *= a1;
#pragma unroll
                            for (int mt = 0; mt < 8; ++mt) {
                                acc[mt][0] *= a0;
                                acc[mt][1] *= a1;
                                acc[mt][2] *= a0;
                                acc[mt][3] *= a1;
                            }
                        }
                        const float mu0 = m_run[0] == -INFINITY ? 0.f : m_run[0];
                        const float mu1 = m_run[1] == -INFINITY ? 0.f : m_run[1];
                        uint32_t bf[MT][2];
#pragma unroll
                        for (int mi = 0; mi < MT; ++mi) {
                            const int row = wt + 16 * mi + rg;
                            const bool ok0 = FULL || 16 * mi + rg < nval, ok1 = FULL || 16 * mi + rg + 8 < nval;
                            const float p0 = fast_exp2(sc[mi][0] - mu0), p1 = fast_exp2(sc[mi][1] - mu1);
                            const float p2 = fast_exp2(sc[mi][2] - mu0), p3 = fast_exp2(sc[mi][3] - mu1);
                            l_run[0] += p0 + p2;
                            l_run[1] += p1 + p3;
                            float v0 = 1.f, v1 = 1.f;  // fp16 V: p is fed as is (0 on masked rows)
                            if constexpr (FMT != kF16) {
                                const __half* svs = reinterpret_cast<const __half*>(sb + p.off_vs);
                                v0 = ok0 ? __half2float(svs[row]) : 0.f;
                                v1 = ok1 ? __half2float(svs[row + 8]) : 0.f;
                            }
                            if (F::ZV) {
                                const __half* svz = reinterpret_cast<const __half*>(sb + p.off_vz);
                                const float z0 = ok0 ? __half2float(svz[row]) : 0.f;
                                const float z1 = ok1 ? __half2float(svz[row + 8]) : 0.f;
                                zv[0] = fmaf(p0, z0, fmaf(p2, z1, zv[0]));
                                zv[1] = fmaf(p1, z0, fmaf(p3, z1, zv[1]));
                            }
                            const uint32_t pr0 = pack_h2(p0 * v0, p1 * v0);
                            const uint32_t pr1 = pack_h2(p2 * v1, p3 * v1);
                            if (!F::ZV && FMT != kF16) {
                                // the exact sum of the fed weights cancels the V code offset
                                fma_h2_2acc(pr0, 0x3c003c00u, lf[0], lf[1]);
                                fma_h2_2acc(pr1, 0x3c003c00u, lf[0], lf[1]);
                            }
                            bf[mi][0] = movmatrix_trans(pr0);
                            bf[mi][1] = movmatrix_trans(pr1);
                        }
                        // ---------------- PV (tensor pipe) ----------------
#pragma unroll
                        for (int mi = 0; mi < MT; ++mi)
                            if (FULL || 16 * mi < nval)
                                pv_kstep<FMT>(sb + p.off_v + (wt + 16 * mi + vr) * ROWB + M::VCB * g,
                                              bf[mi][0], bf[mi][1], acc);
                    }
                }
            };
#pragma unroll 1
            for (int hf = 0; hf < NHALF; ++hf) {
                wt = wt0 + hf * TW;
                nval = aborted ? 0 : ntok - wt;
                if (nval >= TW)
                    tile_body(std::true_type{});
                else
                    tile_body(std::false_type{});
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[st]);
            }  // tile of this warp group

            // ---------------- end of a unit segment ----------------
            if (ti == p.tpu - 1 || i == te - 1) {
                const bool final_seg = (i == te - 1);
                // whole: this CTA's segment covers the unit from its first tile
                const bool whole = (ti == p.tpu - 1) && (unit * p.tpu >= tb);
#pragma unroll
                for (int hh = 0; hh < 2; ++hh)
#pragma unroll
                    for (int m = 4; m < 32; m <<= 1) {
                        l_run[hh] += __shfl_xor_sync(kFull, l_run[hh], m);
                        zv[hh] += __shfl_xor_sync(kFull, zv[hh], m);
                        lf[hh] += __shfl_xor_sync(kFull, lf[hh], m);
                    }
                float* abuf_s = abuf;
                float* mlb_s = mlb;
                if (final_seg) {
                    // The CTA's last segment: every tile is consumed and no copy is
                    // in flight, so once all consumer warps are here the warp states
                    // go into the stage memory, without waiting for the epilogue
                    // warp's hand-off.
                    named_bar_sync(1, kNCW * 32);
                    abuf_s = reinterpret_cast<float*>(smem);
                    mlb_s = abuf_s + kNCW * HB * kHeadDim;
                } else {
                    wait_handoff_free(p, epi_empty, misc, nhand, lane);
                }
#pragma unroll
                for (int hh = 0; hh < 2; ++hh) {
                    const int h = 2 * r + hh;
                    if (h < HB) {
                        if (g == 0) {
                            mlb_s[(w * HB + h) * 3] = m_run[hh];
                            mlb_s[(w * HB + h) * 3 + 1] = l_run[hh];
                        }
                        const float add = F::ZV ? zv[hh] : -M::VOFF * lf[hh];
                        float o[16];
#pragma unroll
                        for (int mt = 0; mt < 8; ++mt) {
                            o[2 * mt] = fmaf(acc[mt][hh], kSub, add);
                            o[2 * mt + 1] = fmaf(acc[mt][2 + hh], kScHi, add);
                        }
                        float4* dst = reinterpret_cast<float4*>(abuf_s + (w * HB + h) * kHeadDim + 16 * g);
#pragma unroll
                        for (int q4 = 0; q4 < 4; ++q4)
                            dst[q4] = make_float4(o[4 * q4], o[4 * q4 + 1], o[4 * q4 + 2], o[4 * q4 + 3]);
                    }
                }
                reset_state();
                const long long bk = p.fd_nhb.q(unit);
                const long long hb = unit - bk * p.nhb;
                const long long b = p.fd_hkv.q(bk);
                const long long kvh = bk - b * p.n_kv_heads;
                const long long qoff = (b * p.n_heads + kvh * p.nhb * HB + hb * HB) * kHeadDim;
                finish_segment<HB>(p, final_seg, whole, unit, qoff, 2 * cta + (unit == first_unit_of_cta ? 0 : 1),
                                   nhand, desc, epi_full, misc, mlb_s, abuf_s, last_span, w, lane, tid);
            }
            if (++st == p.nst) {
                st = 0;
                ph ^= 1u;
            }
            if (++ti == p.tpu) {
                ti = 0;
                ++unit;
            }
        }
        return;
    }

    if constexpr (!MMA) {
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

    uint16_t* pbuf = reinterpret_cast<uint16_t*>(smem + p.off_work) + w * TW * HB;  // p as f16
    const long long first_unit_of_cta = p.fd_tpu.q(tb);
    long long nhand = 0;  // segments handed to the epilogue warp so far
    // span of the CTA's last unit, needed right after its final segment;
    // computed now, while the first tiles are still in flight, and kept in
    // shared memory (read after the final segment's barriers)
    UnitSpan* last_span = reinterpret_cast<UnitSpan*>(smem + p.off_misc + 16 + sizeof(EpiDesc));
    if (tid == 0) *last_span = unit_span(p, p.fd_tpu.q(te - 1));

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
    long long unit = p.fd_tpu.q(tb);
    long long ti = tb - unit * p.tpu;
    for (long long i = tb; i < te; ++i) {
        const bool new_unit = (unit != cur_unit);
        if (new_unit) {
            // ---- start of a unit segment ----
            cur_unit = unit;
            seg_t0 = ti;
            cur_g = -1;
            bk = p.fd_nhb.q(unit);
            const int hb = static_cast<int>(unit - bk * p.nhb);
            const long long b = p.fd_hkv.q(bk);
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

        const long long t0 = ti * T;
        int ntok = static_cast<int>(max(0LL, min(static_cast<long long>(T), seq_len - t0)));
                if (p.paged) ntok = *reinterpret_cast<const volatile int*>(smem + static_cast<size_t>(st) * p.stage_bytes + p.off_ntok);
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
                    const int g0 = static_cast<int>(p.fd_gs.q(t0));
                    gsp = reinterpret_cast<const __half*>(sb + p.off_kgs) + (g - g0) * kHeadDim;
                    if (F::ZK) gzp = reinterpret_cast<const __half*>(sb + p.off_kgz) + (g - g0) * kHeadDim;
                } else {
                    long long gb = (bk * p.ng_buf + g) * kHeadDim;
                    if (p.paged) {
                        const long long pos = static_cast<long long>(g) * p.group_size;
                        const long long sq = p.fd_hkv.q(bk);
                        const long long page = checked_page(p, p.block_tables[sq * p.max_blocks + p.fd_bs.q(pos)]);
                        gb = ((page * p.n_kv_heads + (bk - sq * p.n_kv_heads)) *
                                  p.fd_gs.q(p.block_size) + p.fd_gs.q(p.fd_bs.r(pos))) *
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
                const int g_lo = static_cast<int>(p.fd_gs.q(pos_lo));
                if (g_lo == static_cast<int>(p.fd_gs.q(pos_lo + nval - 1))) {
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
                            if (CHECK && (cur_g < 0 || tabs >= gnext)) load_group(static_cast<int>(p.fd_gs.q(tabs)));
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
            if (PVC == 8) {
#pragma unroll
                for (int h = 0; h < HB; ++h)
#pragma unroll
                    for (int c = 0; c < 8; ++c) acc[h][c] += __shfl_xor_sync(kFull, acc[h][c], 16);
            }
            float* abuf_s = abuf;
            float* mlb_s = mlb;
            if (final_seg) {
                // The CTA's last segment: every tile is consumed and no copy is in
                // flight, so once all consumer warps are here the warp states go into
                // the stage memory, without waiting for the epilogue warp's hand-off.
                named_bar_sync(1, kNCW * 32);
                abuf_s = reinterpret_cast<float*>(smem);
                mlb_s = abuf_s + kNCW * HB * kHeadDim;
            } else {
                wait_handoff_free(p, epi_empty, misc, nhand, lane);
            }
            if (grp == 0 && prim && qpl == 0) {
                mlb_s[(w * HB + hh) * 3] = m_run;
                mlb_s[(w * HB + hh) * 3 + 1] = l_run;
            }
#pragma unroll
            for (int h = 0; h < HB; ++h) {
                float* dst = abuf_s + (w * HB + h) * kHeadDim;
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
            finish_segment<HB>(p, final_seg, whole, unit, qoff, 2 * cta + (unit == first_unit_of_cta ? 0 : 1), nhand,
                               desc, epi_full, misc, mlb_s, abuf_s, last_span, w, lane, tid);
        }
        if (++st == p.nst) {
            st = 0;
            ph ^= 1u;
        }
        if (++ti == p.tpu) {
            ti = 0;
            ++unit;
        }
    }
    }  // !MMA
}

// ---- host side ------------------------------------------------------------

// fp16, INT8 and INT4 run QK / PV on the tensor pipe when no K group
// straddles a 16-position MMA tile (INT4 group sizes that are multiples of
// 16); other INT4 group sizes use the CUDA-core consumer.
bool decode_uses_mma(int fmt, int64_t group_size) {
    return fmt == kF16 || fmt == kI8 || ((fmt == kI4Sym || fmt == kI4Asym) && group_size > 0 && group_size % 16 == 0);
}

int heads_per_unit(int64_t group, int fmt, bool mma) {
    // The tensor-pipe consumer covers eight heads per MMA column block; the
    // CUDA-core INT8/INT4 consumer has registers for four (168 per thread at
    // 10 warps per SM) and splits a group of 8 into two units.
    if (group % 8 == 0 && (fmt == kF16 || mma)) return 8;
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

size_t decode_counter_offset(int sm_count) { return kWsErrBytes + partial_region_bytes(sm_count); }

size_t decode_workspace_bytes(int64_t batch, int64_t n_heads, int64_t n_kv_heads, int sm_count) {
    if (batch <= 0 || n_kv_heads <= 0 || n_heads <= 0) return kWsErrBytes;
    const int64_t n_units = batch * n_heads;  // upper bound over every heads-per-unit choice
    return kWsErrBytes + partial_region_bytes(sm_count) + align_up(static_cast<size_t>(n_units) * 4, 256);
}

namespace {

template <int FMT, int HB, bool MMA>
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
    p.num_blocks = a.num_blocks;
    p.qscale = a.softmax_scale * kLog2e;
    // 32-bit index arithmetic in the kernel (launch-constant divisors)
    if (p.total_tiles >= (int64_t{1} << 31) || a.batch * a.n_kv_heads >= (int64_t{1} << 31)) {
        err = "too many work tiles for one launch (batch * n_heads * seqlen / tile above 2^31)";
        return LIK_ERR_UNSUPPORTED;
    }
    p.fd_tpu = make_fdiv(static_cast<uint32_t>(p.tpu));
    p.fd_nhb = make_fdiv(static_cast<uint32_t>(p.nhb));
    p.fd_hkv = make_fdiv(static_cast<uint32_t>(p.n_kv_heads));
    p.fd_gs = make_fdiv(static_cast<uint32_t>(p.group_size));
    p.fd_bs = make_fdiv(static_cast<uint32_t>(p.block_size > 0 ? p.block_size : 1));

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
    p.off_ntok = off;  // paged: the tile's live length (0 when masked)
    off += 16;
    if (MMA && F::KG) {
        // fixed-point limbs of the folded K weights, per-head score constants
        // and fixed-point steps of the tile's K groups
        p.ngw = static_cast<int>(std::min<int64_t>(a.n_groups_buf, (T + a.group_size - 1) / a.group_size + 1));
        off = static_cast<int>(align_up(off, 16));
        p.off_w = off;
        off += p.ngw * HB * 4 * MmaFmt<FMT>::L * 8 * 4;
        p.off_zk = off;
        off += 2 * p.ngw * HB * 4;
    }
    p.stage_bytes = static_cast<int>(align_up(off, 128));

    // per-warp fp16 softmax weights, then the per-warp raw accumulators
    const int pbuf_bytes =
        MMA ? 0 : static_cast<int>(align_up(static_cast<size_t>(kNCW) * (T / kNCW) * HB * 2, 16));
    const int abuf_bytes = kNCW * HB * kHeadDim * 4;
    // INT4 formats: per-warp score slots (one float per lane and pass group)
    constexpr int kNP = T / kNCW / 4;
    constexpr int kQG = (8 / HB) < kNP ? (8 / HB) : kNP;
    const int sc_bytes = (F::KG && !MMA) ? kNCW * (kNP / kQG) * 32 * 4 : 0;
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
    p.fd_nst = make_fdiv(static_cast<uint32_t>(nst));
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

    auto kern = decode_kernel<FMT, HB, MMA>;
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
    cfg.blockDim = dim3(threads_for<FMT, MMA>());
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

template <int FMT, bool MMA>
lik_status launch_fmt(const DecodeArgs& a, const DeviceInfo& di, cudaStream_t s, std::string& err) {
    switch (heads_per_unit(a.n_heads / a.n_kv_heads, FMT, MMA)) {
        case 8:
            if constexpr (FMT == kF16 || MMA) return launch_t<FMT, 8, MMA>(a, di, s, err);
            err = "internal: eight heads per unit needs the fp16 or tensor-pipe consumer";
            return LIK_ERR_UNSUPPORTED;
        case 4: return launch_t<FMT, 4, MMA>(a, di, s, err);
        case 2: return launch_t<FMT, 2, MMA>(a, di, s, err);
        default: return launch_t<FMT, 1, MMA>(a, di, s, err);
    }
}

}  // namespace

lik_status launch_decode(const DecodeArgs& a, cudaStream_t stream, std::string& err) {
    DeviceInfo di;
    if (!device_info(di, err)) return LIK_ERR_CUDA;
    switch (a.fmt) {
        case kF16: return launch_fmt<kF16, true>(a, di, stream, err);
        case kI8: return launch_fmt<kI8, true>(a, di, stream, err);
        case kI4Sym:
            return decode_uses_mma(a.fmt, a.group_size) ? launch_fmt<kI4Sym, true>(a, di, stream, err)
                                                        : launch_fmt<kI4Sym, false>(a, di, stream, err);
        case kI4Asym:
            return decode_uses_mma(a.fmt, a.group_size) ? launch_fmt<kI4Asym, true>(a, di, stream, err)
                                                        : launch_fmt<kI4Asym, false>(a, di, stream, err);
        default: err = "unknown KV format"; return LIK_ERR_INVALID_ARGUMENT;
    }
}

}  // namespace lik
