// Cell-by-cell filtered beam search: one warp per query, persistent warps pulling
// queries (most cells first) from a device counter.  Re-design of
// select_path_contain_attr_filter_V2_without_output_with_post_pre_filter
// (gpu_graph.cu:3270-4131) and its host driver
// batch_graph_search_gpu_with_prefilter_and_postfilter (gpu_graph.cu:12464-12616).
//
// Per query the warp keeps, in shared memory: the candidate list T (L entries, double
// buffered for rank merges), the recycle list RL (k entries, double buffered), a batch
// buffer B, an eviction buffer, the query row (fp32 pairs), the box bounds, a row
// staging area and a visited hash.  A batch of candidate rows is copied into the staging
// area with cp.async (all rows of an expansion in flight at once, 16-byte coalesced
// segments; the reference keeps six 8-byte loads in flight per query) and each lane then
// computes one candidate's canonical distance from shared memory with packed fp32x2
// arithmetic.  The range predicate is evaluated alongside and kept as a flag bit, so
// evictions and the final filter need no further attribute reads.
#include <algorithm>
#include <random>
#include <vector>
#include <cstdio>

#include "gf_device.cuh"
#include "gf_internal.h"

namespace gf {
namespace {

using namespace dev;

constexpr float kInf = __builtin_huge_valf();

struct SArgs {
    const uint4* __restrict__ vec16;  // stored rows (fp16, or bytes for the byte codecs), 16-byte chunks
    const float* __restrict__ attrs;
    const uint32_t* __restrict__ graph;
    const uint32_t* __restrict__ cross;
    const uint32_t* __restrict__ seg;
    const uint32_t* __restrict__ i2g;
    const uint32_t* __restrict__ spk;  // cross-edge row of each position (spokesman rank), or NULL
    const uint4* __restrict__ q16;
    const float* __restrict__ q32;    // fp32 queries (byte codecs: times alpha, fp32)
    const float* __restrict__ csc;    // byte codecs: per-element -scale (d16)
    const float* __restrict__ cbi;    // byte codecs: per-element 2^23 + bias (d16)
    float alpha;
    uint32_t xmask, dim;
    const float* __restrict__ lb;
    const float* __restrict__ rb;
    const uint32_t* __restrict__ counts;
    const uint32_t* __restrict__ offsets;
    const uint32_t* __restrict__ cells;
    const uint32_t* __restrict__ box;  // box counts (only when prefilter > 0)
    const uint32_t* __restrict__ skip = nullptr;  // queries answered by the tensor-core exact scan
    // attribute tiles of a whole index (exact route without a cell view; NULL: scan the cells)
    const float* __restrict__ sbox = nullptr;   // super-tile bounds (32 tiles each)
    const float* __restrict__ tbox = nullptr;   // tile bounds (128 rows each)
    const float* __restrict__ tattrs = nullptr; // row attributes (NaN past n)
    const uint32_t* __restrict__ trow = nullptr; // row -> position
    uint32_t nstiles = 0, ntiles = 0, a8 = 0;
    const uint32_t* __restrict__ task;
    const uint32_t* __restrict__ entry;
    uint32_t* queue;
    uint32_t* out_ids;
    float* out_d;
    unsigned long long* stats;
    // cell view (NULL slot: every cell, rows at graph + pos*R and cross + pos*P*E + t*E)
    const int32_t* __restrict__ slot;
    const long long* __restrict__ gofs;
    const long long* __restrict__ xofs;
    const long long* __restrict__ vsh;  // per slot: vector row = position + vsh (NULL: 0)
    unsigned long long* run;
    uint32_t nslots, xstride;
    uint32_t qnum, nch, a, P, R, E, L, K, W, max_iter, n_entry, postfilter, n;
    float prefilter;
    uint32_t hs, hshift, bcap, stage_rows, stage_stride, warp_words;
    uint32_t stage_shift;           // log2(stage_rows)
    unsigned long long e_magic;     // ceil(2^32 / E): j / E == (j * e_magic) >> 32 for the hop's pairs
    uint32_t wait_polls, extra_tx;  // staging wait limit; test hook: bytes expected but never sent
    uint32_t graph_bulk;            // neighbour rows are fetched with bulk copies (R * 4 a multiple of 16)
    // word offsets inside a warp's shared-memory slice
    uint32_t o_sc, o_bi;  // byte codecs: -scale and 2^23 + bias pairs
    uint32_t o_q, o_lb, o_rb, o_t0d, o_t0w, o_t1d, o_t1w, o_r0d, o_r0w, o_r1d, o_r1w, o_bd, o_bw, o_ed, o_ew,
        o_picks, o_stage, o_hash, o_mbar;
};

// Shared-memory layout of one warp, in 32-bit words, every region 16-byte aligned.
// Lists hold 64-bit keys (see key_t): T and T' (L each), RL and RL' (k each), the batch B
// and the eviction buffer E (bcap each).  Candidate positions of a batch are gathered
// into E (as 32-bit words) before evaluation, while E is otherwise unused.
void make_layout(SArgs& A, uint32_t nch16, bool bytes) {
    uint32_t o = 0;
    auto take = [&](uint32_t words) {
        uint32_t r = o;
        o += (words + 3) & ~3u;
        return r;
    };
    // fp32 query as (even, odd) element pairs: 4 pairs per fp16 chunk, 8 per byte chunk
    A.o_q = take(nch16 * (bytes ? 16 : 8));
    A.o_sc = bytes ? take(nch16 * 16) : 0;
    A.o_bi = bytes ? take(nch16 * 16) : 0;
    A.o_lb = take(kMaxAttr);
    A.o_rb = take(kMaxAttr);
    A.o_t0d = take(2 * A.L);
    A.o_t1d = take(2 * A.L);
    A.o_r0d = take(2 * A.K);
    A.o_r1d = take(2 * A.K);
    A.o_bd = take(2 * A.bcap);
    A.o_ed = take(2 * A.bcap);
    A.o_t0w = A.o_t1w = A.o_r0w = A.o_r1w = A.o_bw = A.o_ew = 0;
    A.o_picks = take(32);
    A.o_mbar = take(4);  // staging mbarrier (8 bytes), its phase bit, the warp's abort flag
    A.o_stage = take(A.stage_rows * A.stage_stride * 4);
    A.o_hash = take(A.hs);
    A.warp_words = o;
}

// Per-warp view of the shared slice; pointers are recomputed from the base and the
// offsets (kernel parameters) where used, which keeps few registers live.
struct W {
    uint32_t* base;
    uint32_t tsel, rsel;  // which buffer of T / RL is current
    __device__ key_t* T(const SArgs& A) const { return (key_t*)(base + (tsel ? A.o_t1d : A.o_t0d)); }
    __device__ key_t* Tn(const SArgs& A) const { return (key_t*)(base + (tsel ? A.o_t0d : A.o_t1d)); }
    __device__ key_t* RL(const SArgs& A) const { return (key_t*)(base + (rsel ? A.o_r1d : A.o_r0d)); }
    __device__ key_t* RLn(const SArgs& A) const { return (key_t*)(base + (rsel ? A.o_r0d : A.o_r1d)); }
    __device__ key_t* B(const SArgs& A) const { return (key_t*)(base + A.o_bd); }
    __device__ key_t* E(const SArgs& A) const { return (key_t*)(base + A.o_ed); }
    __device__ uint32_t* P(const SArgs& A) const { return base + A.o_ed; }  // batch positions (aliases E)
    __device__ uint32_t* picks(const SArgs& A) const { return base + A.o_picks; }
    __device__ uint32_t* H(const SArgs& A) const { return base + A.o_hash; }
    __device__ const float* lb(const SArgs& A) const { return (const float*)(base + A.o_lb); }
    __device__ const float* rb(const SArgs& A) const { return (const float*)(base + A.o_rb); }
};

__device__ __forceinline__ uint32_t next_pow2(uint32_t x) { return x <= 1 ? 1 : 1u << (32 - __clz(x - 1)); }

// Bounded wait for a staging batch: polls of the mbarrier before the warp gives up,
// counts a timeout in stats[7] and stops evaluating (the host reports GF_ERR_TIMEOUT).
constexpr uint32_t kStageWaitPolls = 1u << 19;  // with the suspend hint, about a second
constexpr uint32_t kStageSuspendNs = 2000;  // suspend hint of each poll (a copy takes ~1-3 us)

// Bounded wait for the copies counted on the warp's staging mbarrier, then the phase bit
// flips.  A wait that runs out stops the warp: the abort flag is set, stats[7] counts it
// and true is returned (the staging buffers are not used again by this warp).
__device__ __forceinline__ bool stage_wait(const SArgs& A, uint32_t* base) {
    uint64_t* bar = reinterpret_cast<uint64_t*>(base + A.o_mbar);
    uint32_t* phase = base + A.o_mbar + 2;
    const uint32_t par = *phase;
    uint32_t polls = 0;
    while (!mbar_try_wait(bar, par, kStageSuspendNs) && ++polls < A.wait_polls) {
    }
    const bool timed_out = __any_sync(kFull, polls >= A.wait_polls);
    __syncwarp();
    if (lane_id() == 0) {
        *phase = par ^ 1u;
        if (timed_out) {
            base[A.o_mbar + 3] = 1u;
            atomicAdd(A.stats + 7, 1ull);
        }
    }
    __syncwarp();
    return timed_out;
}

// Distances + range flags of the positions P[0..nb); the keys below `thr` (the list's
// worst entry, or kEmptyKey for no bound) are written sorted to B[0..ns), padded with
// empty keys to a power of two >= 32; returns ns.  A key at or above the list's worst
// entry cannot enter the list, so dropping it before the sort leaves every merge result
// unchanged.  Rows are staged through shared memory stage_rows (<= 16) at a time, one bulk
// (TMA) copy per row, completion on the warp's mbarrier.  Staged rows lie stage_stride chunks apart (an odd number, so lanes reading the same chunk of consecutive rows hit
// different bank groups).  Lanes r and r + 16 evaluate row r, one chunk parity each, and
// lane r adds the two halves.  At most 32 survivors are sorted in registers, more in
// shared memory.  Kept out of line: one copy of the distance loop and
// sort network serves the entry set, the beam rounds, the hop and the exact route.
template <int NCH, bool BYTES>
__device__ __noinline__ uint32_t eval_sort(const SArgs& A, uint32_t* base, uint32_t nb, key_t thr, long long vsh) {
    const W w{base, 0u, 0u};
    const uint32_t lane = lane_id();
    const uint32_t nch = NCH ? (uint32_t)NCH : A.nch;
    const uint32_t stride = A.stage_stride, row_bytes = nch * 16;
    const uint32_t* P = w.P(A);
    key_t* B = w.B(A);
    uint4* stage = reinterpret_cast<uint4*>(w.base + A.o_stage);
    uint64_t* bar = reinterpret_cast<uint64_t*>(w.base + A.o_mbar);
    uint32_t* abort = w.base + A.o_mbar + 3;
    const f2x* q2 = reinterpret_cast<const f2x*>(w.base + A.o_q);
    const uint32_t SR = A.stage_rows, row = lane & 15u, half = lane >> 4;
    uint32_t ns = 0;
    if (*abort) return 0;
    // copies of stage s (rows s*SR ..); returns the lane's in-range flag
    auto issue = [&](uint32_t s) -> bool {
        const uint32_t r0 = s * SR, rows = min(SR, nb - r0);
        fence_proxy_async_smem();  // earlier reads of the staging area come before the copies
        __syncwarp();
        if (lane == 0) mbar_arrive_expect_tx(bar, rows * row_bytes + A.extra_tx);
        __syncwarp();
        bool inr = false;
        if (lane < rows) {
            const uint32_t pos = P[r0 + lane];
            bulk_g2s(stage + (size_t)lane * stride, A.vec16 + (pos + vsh) * nch, row_bytes, bar);
            inr = in_box(A.attrs, pos, A.a, w.lb(A), w.rb(A));
        }
        return inr;
    };
    const uint32_t nst = (nb + SR - 1) >> A.stage_shift;
    bool inr_next = nst ? issue(0) : false;
    for (uint32_t s = 0; s < nst; ++s) {
        const bool inr = inr_next;
        const uint32_t r0 = s * SR, rows = min(SR, nb - r0);
        if (stage_wait(A, w.base)) return 0;
        f2x acc[4] = {0ull, 0ull, 0ull, 0ull};
        if (row < rows) {
            const uint4* srow = stage + (size_t)row * stride;
            if (BYTES)
                half8<NCH>(srow, q2, reinterpret_cast<const f2x*>(w.base + A.o_sc),
                           reinterpret_cast<const f2x*>(w.base + A.o_bi), A.xmask, nch, half, acc);
            else
                half16<NCH>(srow, q2, nch, half, acc);
        }
#pragma unroll
        for (int m = 0; m < 4; ++m) acc[m] = add2(acc[m], __shfl_down_sync(kFull, acc[m], 16));
        key_t k = kEmptyKey;
        if (lane < rows) k = make_key(finish8(acc[0], acc[1], acc[2], acc[3]), P[r0 + lane], inr ? kKeyInRange : 0u);
        const bool keep = k < thr;
        const uint32_t msk = __ballot_sync(kFull, keep);
        if (keep) B[ns + __popc(msk & lanemask_lt())] = k;
        ns += __popc(msk);
        __syncwarp();
        if (s + 1 < nst) inr_next = issue(s + 1);
    }
    if (ns <= 32) {
        if (ns) {
            const key_t k = lane < ns ? B[lane] : kEmptyKey;
            __syncwarp();
            B[lane] = warp_sort_key_upto(k, next_pow2(ns));
            __syncwarp();
        }
        return ns;
    }
    const uint32_t n = next_pow2(ns);
    for (uint32_t j = ns + lane; j < n; j += 32) B[j] = kEmptyKey;
    __syncwarp();
    warp_sort_keys(B, n);
    return ns;
}

// Merge B[b0..b0+nb) into T (length L); with recycling, in-range entries pushed out of
// T are merged into RL (length k).
__device__ __forceinline__ void merge_step(const SArgs& A, W& w, uint32_t L, uint32_t b0, uint32_t nb, bool recycle) {
    if (nb == 0) return;
    const key_t* B = w.B(A) + b0;
    {
        const key_t last = w.T(A)[L - 1];
        // nothing can enter a full list whose last entry beats the best candidate
        if (last != kEmptyKey && B[0] > last) return;
    }
    const uint32_t r = merge_keys(w.T(A), w.Tn(A), L, B, nb, w.E(A), recycle);
    if ((r >> 16) == 0) return;
    w.tsel ^= 1u;
    const uint32_t nev = r & 0xFFFFu;
    if (nev == 0) return;
    const key_t rlast = w.RL(A)[A.K - 1];
    if (rlast != kEmptyKey && w.E(A)[0] > rlast) return;
    const uint32_t r2 = merge_keys(w.RL(A), w.RLn(A), A.K, w.E(A), nev, nullptr, false);
    if ((r2 >> 16) != 0) w.rsel ^= 1u;
}

// Clear the hash and insert the list entries that lie in [lo, hi); returns how many.
__device__ __forceinline__ uint32_t hash_rebuild(const SArgs& A, const W& w, uint32_t lo, uint32_t hi) {
    uint32_t* H = w.H(A);
    const key_t* T = w.T(A);
    hash_clear(H, A.hs);
    uint32_t cnt = 0;
    for (uint32_t i0 = 0; i0 < A.L; i0 += 32) {
        uint32_t i = i0 + lane_id();
        bool ins = false;
        if (i < A.L) {
            const key_t k = T[i];
            const uint32_t pos = key_pos(k);
            if (k != kEmptyKey && pos >= lo && pos < hi) ins = hash_insert(H, A.hs, A.hshift, pos);
        }
        cnt += __popc(__ballot_sync(kFull, ins));
    }
    __syncwarp();
    return cnt;
}

__device__ __forceinline__ void write_result(const SArgs& A, uint32_t q, const key_t* list, uint32_t n) {
    for (uint32_t k = lane_id(); k < A.K; k += 32) {
        const key_t v = k < n ? list[k] : kEmptyKey;
        A.out_ids[(size_t)q * A.K + k] = v == kEmptyKey ? kEmpty : A.i2g[key_pos(v)];
        if (A.out_d) A.out_d[(size_t)q * A.K + k] = v == kEmptyKey ? kInf : key_dist(v);
    }
}

// Result of query q: the sorted k-list `res` is written as ids, or, under a cell view,
// merged into the query's running keys run[q] (ta, tb: k-key scratch lists).
__device__ __noinline__ void emit(const SArgs& A, uint32_t q, const key_t* res, key_t* ta, key_t* tb) {
    if (!A.run) {
        write_result(A, q, res, A.K);
        return;
    }
    const uint32_t lane = lane_id();
    unsigned long long* rq = A.run + (size_t)q * A.K;
    uint32_t nres = 0;
    for (uint32_t i0 = 0; i0 < A.K; i0 += 32) {
        const uint32_t i = i0 + lane;
        nres += __popc(__ballot_sync(kFull, i < A.K && res[i] != kEmptyKey));
    }
    if (nres == 0) return;
    for (uint32_t i = lane; i < A.K; i += 32) ta[i] = rq[i];
    __syncwarp();
    const uint32_t r = merge_keys(ta, tb, A.K, res, nres, nullptr, false);
    if ((r >> 16) == 0) return;
    for (uint32_t i = lane; i < A.K; i += 32) rq[i] = tb[i];
}

// Row offset of a cell's stored vectors: row = position + cell_vsh.
__device__ __forceinline__ long long cell_vsh(const SArgs& A, uint32_t cell) {
    return A.vsh ? A.vsh[A.slot[cell]] : 0ll;
}

// Index in cl[0..nc) of the first cell at or after ci that this launch searches.
__device__ __forceinline__ uint32_t next_cell(const SArgs& A, const uint32_t* cl, uint32_t nc, uint32_t ci) {
    if (A.slot)
        while (ci < nc && A.slot[cl[ci]] < 0) ++ci;
    return ci;
}

// Element offset from A.graph of the row of position p in `cell` (seg start lo) is
// gbase + p * R.
__device__ __forceinline__ long long graph_base(const SArgs& A, uint32_t cell, uint32_t lo) {
    return A.slot ? A.gofs[A.slot[cell]] - (long long)lo * A.R : 0ll;
}

// Element offset from A.cross of the cross edges of position src toward cell `next`.
__device__ __forceinline__ long long cross_row(const SArgs& A, uint32_t src, uint32_t next) {
    if (!A.slot) {
        // spokesman-compressed edges: the row of the point's spokesman
        const uint32_t row = A.spk ? __ldg(A.spk + src) : src;
        return (long long)row * A.P * A.E + (long long)next * A.E;
    }
    uint32_t lo = 0, hi = A.P;  // A.seg[lo] <= src < A.seg[hi]
    while (hi - lo > 1) {
        const uint32_t mid = (lo + hi) >> 1;
        if (A.seg[mid] <= src)
            lo = mid;
        else
            hi = mid;
    }
    // xofs[target slot][source slot] is the block's start less its first row times xstride;
    // a source row is the position, or its spokesman's rank with compressed cross edges
    const uint32_t row = A.spk ? __ldg(A.spk + src) : src;
    return A.xofs[(long long)A.slot[next] * A.nslots + A.slot[lo]] + (long long)row * A.xstride;
}

// Append the positions held by lanes with ok=true to P at nb (warp-uniform counter).
__device__ __forceinline__ void append(uint32_t* P, uint32_t& nb, bool ok, uint32_t pos) {
    uint32_t msk = __ballot_sync(kFull, ok);
    if (ok) P[nb + __popc(msk & lanemask_lt())] = pos;
    nb += __popc(msk);
}

// Neighbour rows of the np picks into G with plain loads (graphs whose rows are not a
// multiple of 16 bytes; others use one bulk copy per row).
__device__ __noinline__ void copy_rows(const SArgs& A, uint32_t* G, const uint32_t* picks, uint32_t np,
                                       long long gbase) {
    for (uint32_t j = lane_id(); j < np * A.R; j += 32)
        G[j] = __ldg(A.graph + (gbase + (long long)picks[j / A.R] * A.R + (j % A.R)));
    __syncwarp();
}

// Exact route (gpu_graph.cu:3788-4022): every in-range point of the query's cells.
template <int NCH, bool BYTES>
__device__ __noinline__ uint32_t exact_route(const SArgs& A, uint32_t* base, uint32_t q, const uint32_t* cl,
                                             uint32_t nc) {
    const uint32_t lane = lane_id();
    W w{base, 0u, 0u};
    for (uint32_t i = lane; i < A.K; i += 32) w.T(A)[i] = kEmptyKey;
    __syncwarp();
    uint32_t nb = 0, ndist = 0;
    const uint32_t flush_at = A.bcap - 32;
    if (A.tbox) {
        // whole index: the in-box points are found through the attribute tiles (super-tiles,
        // then tiles that meet the box, then their rows) instead of every row of the cells.
        // The same points are evaluated with the same distances, and the K smallest keys do
        // not depend on the order, so the result is the cell scan's.
        const float* lb = w.lb(A);
        const float* rb = w.rb(A);
        auto meets = [&](const float* b) {
            bool m = true;
            for (uint32_t j = 0; j < A.a; ++j) m = m && (b[j] <= rb[j]) && (lb[j] <= b[A.a8 + j]);
            return m;
        };
        for (uint32_t s0 = 0; s0 < A.nstiles; s0 += 32) {
            const uint32_t st = s0 + lane;
            uint32_t ps = __ballot_sync(kFull, st < A.nstiles && meets(A.sbox + (size_t)st * 2 * A.a8));
            while (ps) {
                const uint32_t ss = s0 + __ffs(ps) - 1;
                ps &= ps - 1;
                const uint32_t t = ss * kSuperTiles + lane;
                uint32_t pt = __ballot_sync(kFull, t < A.ntiles && meets(A.tbox + (size_t)t * 2 * A.a8));
                while (pt) {
                    const uint32_t tt = ss * kSuperTiles + __ffs(pt) - 1;
                    pt &= pt - 1;
                    for (uint32_t g = 0; g < kTileRows / 32; ++g) {
                        const uint32_t r = tt * kTileRows + g * 32 + lane;
                        const bool ok = in_box(A.tattrs, r, A.a, lb, rb);  // NaN rows (padding) never
                        append(w.P(A), nb, ok, ok ? __ldg(A.trow + r) : 0u);
                        if (nb > flush_at) {
                            __syncwarp();
                            const uint32_t ns = eval_sort<NCH, BYTES>(A, w.base, nb, w.T(A)[A.K - 1], 0ll);
                            ndist += nb;
                            merge_step(A, w, A.K, 0, ns, false);
                            nb = 0;
                        }
                    }
                }
            }
        }
        if (nb) {
            __syncwarp();
            const uint32_t ns = eval_sort<NCH, BYTES>(A, w.base, nb, w.T(A)[A.K - 1], 0ll);
            ndist += nb;
            merge_step(A, w, A.K, 0, ns, false);
            nb = 0;
        }
    }
    for (uint32_t ci = A.tbox ? nc : next_cell(A, cl, nc, 0); ci < nc;) {
        const uint32_t cell = cl[ci], lo = A.seg[cell], hi = A.seg[cell + 1];
        const uint32_t cn = next_cell(A, cl, nc, ci + 1);
        const long long vsh = cell_vsh(A, cell);
        for (uint32_t x0 = lo; x0 < hi; x0 += 32) {
            const uint32_t x = x0 + lane;
            append(w.P(A), nb, x < hi && in_box(A.attrs, x, A.a, w.lb(A), w.rb(A)), x);
            const bool last = x0 + 32 >= hi;  // batches never span cells (rows are per cell)
            if (nb > flush_at || (last && nb)) {
                __syncwarp();
                const uint32_t ns = eval_sort<NCH, BYTES>(A, w.base, nb, w.T(A)[A.K - 1], vsh);
                ndist += nb;
                merge_step(A, w, A.K, 0, ns, false);
                nb = 0;
            }
        }
        ci = cn;
    }
    __syncwarp();
    emit(A, q, w.T(A), w.RL(A), w.RLn(A));
    return ndist;
}

// Cross-cell hop into cell `next` (gpu_graph.cu:3564-3643): the distinct cross-edge
// targets of the first min(L, 64) list entries plus the smallest unused local ids of
// the next cell as filler are evaluated and sorted; the first n_entry become the next
// entry set (left sorted in B[0..ne)), the following 64 are merged into T without
// recycling.  Rebuilds the visited hash for the next cell.  Returns ne; adds to stats.
template <int NCH, bool BYTES>
__device__ __noinline__ uint32_t cross_hop(const SArgs& A, W& w, uint32_t next, uint32_t& hcount, uint32_t& st_dist,
                                           uint32_t& st_cross) {
    const uint32_t lane = lane_id();
    const uint32_t nlo = A.seg[next], nsz = A.seg[next + 1] - nlo;
    const uint32_t hop_n = A.L < kHopSlots ? A.L : kHopSlots;
    const key_t* T = w.T(A);
    uint32_t V = 0;
    for (uint32_t i0 = 0; i0 < hop_n; i0 += 32) {
        uint32_t i = i0 + lane;
        V += __popc(__ballot_sync(kFull, i < hop_n && T[i] != kEmptyKey));
    }
    uint32_t* H = w.H(A);
    hash_clear(H, A.hs);
    const uint32_t pairs = V * A.E;
    uint32_t nb = 0;
    uint32_t* P = w.P(A);
    for (uint32_t j0 = 0; j0 < pairs; j0 += 32) {
        uint32_t j = j0 + lane;
        bool ok = false;
        uint32_t pos = kEmpty;
        if (j < pairs) {
            const uint32_t si = (uint32_t)(((unsigned long long)j * A.e_magic) >> 32);  // j / E
            const uint32_t src = key_pos(T[si]);
            pos = __ldg(A.cross + cross_row(A, src, next) + (j - si * A.E));
            if (pos != kEmpty) ok = hash_insert(H, A.hs, A.hshift, pos);
        }
        append(P, nb, ok, pos);
    }
    __syncwarp();
    st_cross += V;
    // filler: smallest local ids of the next cell not among the targets
    uint32_t nf = pairs - nb;
    for (uint32_t x0 = 0; nf > 0 && x0 < nsz; x0 += 32) {
        uint32_t x = x0 + lane;
        bool ok = x < nsz && !hash_contains(H, A.hs, A.hshift, nlo + x);
        uint32_t msk = __ballot_sync(kFull, ok);
        uint32_t idx = __popc(msk & lanemask_lt());
        if (ok && idx < nf) P[nb + idx] = nlo + x;
        uint32_t take = min((uint32_t)__popc(msk), nf);
        nb += take;
        nf -= take;
    }
    __syncwarp();
    // every key is below kEmptyKey, so ns == nb unless the warp stopped on a staging timeout
    const uint32_t ns = eval_sort<NCH, BYTES>(A, w.base, nb, kEmptyKey, cell_vsh(A, next));
    st_dist += nb;
    const uint32_t ne = min(ns, A.n_entry);
    const uint32_t nm = min(ns - ne, kHopSlots);
    merge_step(A, w, A.L, ne, nm, false);
    // visited set of the next cell: its entry set + its points now in T
    hash_clear(H, A.hs);
    const key_t* B = w.B(A);
    uint32_t cnt = 0;
    for (uint32_t i0 = 0; i0 < ne; i0 += 32) {
        uint32_t i = i0 + lane;
        bool ins = i < ne && hash_insert(H, A.hs, A.hshift, key_pos(B[i]));
        cnt += __popc(__ballot_sync(kFull, ins));
    }
    const key_t* T2 = w.T(A);
    for (uint32_t i0 = 0; i0 < A.L; i0 += 32) {
        uint32_t i = i0 + lane;
        bool ins = false;
        if (i < A.L) {
            const key_t k = T2[i];
            const uint32_t pos = key_pos(k);
            if (k != kEmptyKey && pos >= nlo && pos < nlo + nsz) ins = hash_insert(H, A.hs, A.hshift, pos);
        }
        cnt += __popc(__ballot_sync(kFull, ins));
    }
    __syncwarp();
    hcount = cnt;
    return ne;
}

template <int NCH, bool BYTES>
__global__ void __launch_bounds__(128, 5) gmg_search_kernel(const __grid_constant__ SArgs A) {
    extern __shared__ __align__(16) uint32_t smem[];
    const uint32_t lane = lane_id();
    uint32_t* const base = smem + (threadIdx.x >> 5) * A.warp_words;
    const uint32_t nch = NCH ? (uint32_t)NCH : A.nch;
    if (lane == 0) {
        mbar_init(reinterpret_cast<uint64_t*>(base + A.o_mbar), 1);
        base[A.o_mbar + 2] = 0;  // phase
        base[A.o_mbar + 3] = 0;  // abort
        fence_mbar_init();
    }
    __syncwarp();

    for (;;) {
        uint32_t slot = 0;
        if (lane == 0) slot = atomicAdd(A.queue, 1u);
        slot = __shfl_sync(kFull, slot, 0);
        if (slot >= A.qnum) break;
        const uint32_t q = A.task[slot];
        if (A.skip && A.skip[q]) continue;  // answered by the tensor-core exact scan
        const uint32_t nc = A.counts[q];
        const uint32_t* cl = A.cells + A.offsets[q];
        // query row (fp16 -> fp32 element pairs) and box
        {
            if (BYTES) {
                float* qf = reinterpret_cast<float*>(base + A.o_q);
                float* sc = reinterpret_cast<float*>(base + A.o_sc);
                float* bi = reinterpret_cast<float*>(base + A.o_bi);
                for (uint32_t i = lane; i < nch * 16; i += 32) {
                    qf[i] = i < A.dim ? __fmul_rn(A.q32[(size_t)q * A.dim + i], A.alpha) : 0.0f;
                    sc[i] = A.csc[i];
                    bi[i] = A.cbi[i];
                }
            } else {
                f2x* q2 = reinterpret_cast<f2x*>(base + A.o_q);
                for (uint32_t c = lane; c < nch; c += 32) {
                    const uint4 v = A.q16[(size_t)q * nch + c];
                    q2[c * 4 + 0] = h2_to_f2x(v.x);
                    q2[c * 4 + 1] = h2_to_f2x(v.y);
                    q2[c * 4 + 2] = h2_to_f2x(v.z);
                    q2[c * 4 + 3] = h2_to_f2x(v.w);
                }
            }
            if (lane < A.a) {
                base[A.o_lb + lane] = __float_as_uint(A.lb[(size_t)q * A.a + lane]);
                base[A.o_rb + lane] = __float_as_uint(A.rb[(size_t)q * A.a + lane]);
            }
            __syncwarp();
        }
        uint32_t st_dist = 0, st_exp = 0, st_cross = 0, st_hops = 0, st_exact = 0;
        const uint32_t c0 = next_cell(A, cl, nc, 0);
        if (c0 == nc) {
            if (!A.run) write_result(A, q, nullptr, 0);
        } else {
            bool exact = nc >= A.postfilter;
            if (!exact && A.box) {
                float prop = (float)((double)A.box[q] / (double)A.n);  // real_dataset_adapter.cuh:380
                exact = prop <= A.prefilter;
            }
            if (exact) {
                st_exact = 1;
                st_dist = exact_route<NCH, BYTES>(A, base, q, cl, nc);
            } else {
                W w{base, 0u, 0u};
                for (uint32_t i = lane; i < A.L; i += 32) w.T(A)[i] = kEmptyKey;
                for (uint32_t i = lane; i < A.K; i += 32) w.RL(A)[i] = kEmptyKey;
                hash_clear(w.H(A), A.hs);
                uint32_t hcount = 0;
                // entry set of the first cell (gpu_graph.cu:3347-3351)
                uint32_t nb = 0;
                {
                    const uint32_t cell = cl[c0], lo = A.seg[cell], sz = A.seg[cell + 1] - lo;
                    for (uint32_t i0 = 0; i0 < A.n_entry; i0 += 32) {
                        uint32_t i = i0 + lane;
                        bool ok = false;
                        uint32_t pos = 0;
                        if (i < A.n_entry) {
                            uint32_t e = A.entry[i];
                            if (e < sz) {
                                pos = lo + e;
                                ok = hash_insert(w.H(A), A.hs, A.hshift, pos);
                            }
                        }
                        append(w.P(A), nb, ok, pos);
                    }
                    __syncwarp();
                    hcount = nb;
                    // ns == nb unless the warp stopped on a staging timeout
                    const uint32_t n0 = nb;
                    nb = eval_sort<NCH, BYTES>(A, w.base, n0, kEmptyKey, cell_vsh(A, cell));
                    st_dist += n0;
                }
                for (uint32_t ci = c0; ci < nc;) {
                    const uint32_t cell = cl[ci], lo = A.seg[cell], hi = A.seg[cell + 1];
                    const long long gbase = graph_base(A, cell, lo);
                    const long long vsh = cell_vsh(A, cell);
                    // (a) entry set -> T, with recycling
                    merge_step(A, w, A.L, 0, nb, true);
                    // (b) beam rounds: expand the first W unexplored entries of T
                    for (uint32_t it = 0; it < A.max_iter; ++it) {
                        uint32_t np = 0;
                        {
                            key_t* T = w.T(A);
                            uint32_t* picks = w.picks(A);
                            // the first W unexplored entries in list order: each lane's rank
                            // among them is a prefix count of the ballot
                            for (uint32_t i0 = 0; i0 < A.L && np < A.W; i0 += 32) {
                                const uint32_t i = i0 + lane;
                                const key_t k = i < A.L ? T[i] : kEmptyKey;
                                const bool fresh = (k & kKeyExplored) == 0;
                                const uint32_t msk = __ballot_sync(kFull, fresh);
                                const uint32_t r = np + __popc(msk & lanemask_lt());
                                if (fresh && r < A.W) {
                                    T[i] = k | kKeyExplored;
                                    picks[r] = key_pos(k);
                                }
                                np = min(np + __popc(msk), A.W);
                            }
                            __syncwarp();
                        }
                        if (np == 0) break;
                        st_exp += np;
                        const uint32_t total = np * A.R;
                        if (hcount + total > (A.hs >> 1)) hcount = hash_rebuild(A, w, lo, hi);
                        nb = 0;
                        {
                            const uint32_t* picks = w.picks(A);
                            uint32_t* H = w.H(A);
                            // the picks' neighbour rows, staged in B (free between a merge
                            // and the next evaluation): one bulk copy per row and one wait
                            uint32_t* G = reinterpret_cast<uint32_t*>(w.B(A));
                            bool have = !w.base[A.o_mbar + 3];
                            if (have) {
                                if (A.graph_bulk) {
                                    fence_proxy_async_smem();
                                    __syncwarp();
                                    if (lane == 0)
                                        mbar_arrive_expect_tx(reinterpret_cast<uint64_t*>(w.base + A.o_mbar),
                                                              np * A.R * 4 + A.extra_tx);
                                    __syncwarp();
                                    if (lane < np)
                                        bulk_g2s(G + lane * A.R, A.graph + (gbase + (long long)picks[lane] * A.R),
                                                 A.R * 4, reinterpret_cast<uint64_t*>(w.base + A.o_mbar));
                                    have = !stage_wait(A, w.base);
                                } else {
                                    copy_rows(A, G, picks, np, gbase);
                                }
                            }
                            if (have) {
                                for (uint32_t j0 = 0; j0 < total; j0 += 32) {
                                    const uint32_t j = j0 + lane;
                                    bool ok = false;
                                    uint32_t pos = kEmpty;
                                    if (j < total) {
                                        pos = G[j];
                                        if (pos != kEmpty) ok = hash_insert(H, A.hs, A.hshift, pos);
                                    }
                                    append(w.P(A), nb, ok, pos);
                                }
                            }
                            __syncwarp();
                        }
                        hcount += nb;
                        if (nb == 0) continue;
                        const uint32_t ns = eval_sort<NCH, BYTES>(A, w.base, nb, w.T(A)[A.L - 1], vsh);
                        st_dist += nb;
                        merge_step(A, w, A.L, 0, ns, true);
                    }
                    // (c) everything in T counts as explored from here on
                    {
                        key_t* T = w.T(A);
                        for (uint32_t i = lane; i < A.L; i += 32) T[i] |= kKeyExplored;
                        __syncwarp();
                    }
                    // (d) cross-cell hop
                    const uint32_t cn = next_cell(A, cl, nc, ci + 1);
                    if (cn < nc) {
                        nb = cross_hop<NCH, BYTES>(A, w, cl[cn], hcount, st_dist, st_cross);
                        ++st_hops;
                    }
                    ci = cn;
                }
                // final post-filter of T and recycle merge (gpu_graph.cu:4025-4048)
                uint32_t nin = 0;
                {
                    const key_t* T = w.T(A);
                    key_t* Tn = w.Tn(A);
                    for (uint32_t i0 = 0; i0 < A.L; i0 += 32) {
                        uint32_t i = i0 + lane;
                        key_t k = i < A.L ? T[i] : kEmptyKey;
                        bool ok = k != kEmptyKey && (k & kKeyInRange);
                        uint32_t msk = __ballot_sync(kFull, ok);
                        if (ok) Tn[nin + __popc(msk & lanemask_lt())] = k;
                        nin += __popc(msk);
                    }
                    __syncwarp();
                }
                const key_t* res = w.RL(A);
                if (nin) {
                    const uint32_t r = merge_keys(w.RL(A), w.RLn(A), A.K, w.Tn(A), nin, nullptr, false);
                    if ((r >> 16) != 0) res = w.RLn(A);
                }
                emit(A, q, res, w.T(A), w.Tn(A));
            }
        }
        __syncwarp();
        if (lane == 0) {
            atomicAdd(A.stats + 0, (unsigned long long)st_dist);
            atomicAdd(A.stats + 1, (unsigned long long)st_exp);
            atomicAdd(A.stats + 2, (unsigned long long)st_cross);
            atomicAdd(A.stats + 3, (unsigned long long)st_hops);
            atomicAdd(A.stats + 4, (unsigned long long)st_exact);
            atomicAdd(A.stats + 5, 1ull);
        }
    }
}

// Full-graph post-filter search (full_graph_search_postfiltering, full_graph_search.cuh:
// 179-593): the same warp-per-query beam rounds as gmg_search_kernel, over the assembled
// graph (A.graph, A.R entries per row) of the whole index -- no cell walk, no hops, no
// recycle list; the box is applied once, to the final list.  Entry set: A.entry holds
// positions.
template <int NCH, bool BYTES>
__global__ void __launch_bounds__(128, 5) fullgraph_kernel(const __grid_constant__ SArgs A) {
    extern __shared__ __align__(16) uint32_t smem[];
    const uint32_t lane = lane_id();
    uint32_t* const base = smem + (threadIdx.x >> 5) * A.warp_words;
    const uint32_t nch = NCH ? (uint32_t)NCH : A.nch;
    if (lane == 0) {
        mbar_init(reinterpret_cast<uint64_t*>(base + A.o_mbar), 1);
        base[A.o_mbar + 2] = 0;
        base[A.o_mbar + 3] = 0;
        fence_mbar_init();
    }
    __syncwarp();
    for (;;) {
        uint32_t slot = 0;
        if (lane == 0) slot = atomicAdd(A.queue, 1u);
        slot = __shfl_sync(kFull, slot, 0);
        if (slot >= A.qnum) break;
        const uint32_t q = A.task[slot];
        if (BYTES) {
            float* qf = reinterpret_cast<float*>(base + A.o_q);
            float* sc = reinterpret_cast<float*>(base + A.o_sc);
            float* bi = reinterpret_cast<float*>(base + A.o_bi);
            for (uint32_t i = lane; i < nch * 16; i += 32) {
                qf[i] = i < A.dim ? __fmul_rn(A.q32[(size_t)q * A.dim + i], A.alpha) : 0.0f;
                sc[i] = A.csc[i];
                bi[i] = A.cbi[i];
            }
        } else {
            f2x* q2 = reinterpret_cast<f2x*>(base + A.o_q);
            for (uint32_t c = lane; c < nch; c += 32) {
                const uint4 v = A.q16[(size_t)q * nch + c];
                q2[c * 4 + 0] = h2_to_f2x(v.x);
                q2[c * 4 + 1] = h2_to_f2x(v.y);
                q2[c * 4 + 2] = h2_to_f2x(v.z);
                q2[c * 4 + 3] = h2_to_f2x(v.w);
            }
        }
        if (lane < A.a) {
            base[A.o_lb + lane] = __float_as_uint(A.lb[(size_t)q * A.a + lane]);
            base[A.o_rb + lane] = __float_as_uint(A.rb[(size_t)q * A.a + lane]);
        }
        __syncwarp();
        uint32_t st_dist = 0, st_exp = 0;
        W w{base, 0u, 0u};
        for (uint32_t i = lane; i < A.L; i += 32) w.T(A)[i] = kEmptyKey;
        hash_clear(w.H(A), A.hs);
        uint32_t nb = 0;
        for (uint32_t i0 = 0; i0 < A.n_entry; i0 += 32) {
            const uint32_t i = i0 + lane;
            bool ok = false;
            uint32_t pos = 0;
            if (i < A.n_entry) {
                pos = A.entry[i];
                ok = pos < A.n && hash_insert(w.H(A), A.hs, A.hshift, pos);
            }
            append(w.P(A), nb, ok, pos);
        }
        __syncwarp();
        uint32_t hcount = nb;
        {
            const uint32_t n0 = nb;
            nb = eval_sort<NCH, BYTES>(A, w.base, n0, kEmptyKey, 0);
            st_dist += n0;
        }
        merge_step(A, w, A.L, 0, nb, false);
        for (uint32_t it = 0; it < A.max_iter; ++it) {
            uint32_t np = 0;
            {
                key_t* T = w.T(A);
                uint32_t* picks = w.picks(A);
                for (uint32_t i0 = 0; i0 < A.L && np < A.W; i0 += 32) {
                    const uint32_t i = i0 + lane;
                    const key_t k = i < A.L ? T[i] : kEmptyKey;
                    uint32_t msk = __ballot_sync(kFull, (k & kKeyExplored) == 0);
                    while (msk && np < A.W) {
                        const uint32_t b = __ffs(msk) - 1;
                        msk &= msk - 1;
                        if (lane == b) {
                            T[i] = k | kKeyExplored;
                            picks[np] = key_pos(k);
                        }
                        ++np;
                    }
                }
                __syncwarp();
            }
            if (np == 0) break;
            st_exp += np;
            const uint32_t total = np * A.R;
            if (hcount + total > (A.hs >> 1)) hcount = hash_rebuild(A, w, 0, A.n);
            nb = 0;
            {
                const uint32_t* picks = w.picks(A);
                uint32_t* H = w.H(A);
                uint32_t* G = reinterpret_cast<uint32_t*>(w.B(A));
                bool have = !w.base[A.o_mbar + 3];
                if (have) {
                    if (A.graph_bulk) {
                        fence_proxy_async_smem();
                        __syncwarp();
                        if (lane == 0)
                            mbar_arrive_expect_tx(reinterpret_cast<uint64_t*>(w.base + A.o_mbar),
                                                  np * A.R * 4 + A.extra_tx);
                        __syncwarp();
                        if (lane < np)
                            bulk_g2s(G + lane * A.R, A.graph + (long long)picks[lane] * A.R, A.R * 4,
                                     reinterpret_cast<uint64_t*>(w.base + A.o_mbar));
                        have = !stage_wait(A, w.base);
                    } else {
                        copy_rows(A, G, picks, np, 0);
                    }
                }
                if (have) {
                    for (uint32_t j0 = 0; j0 < total; j0 += 32) {
                        const uint32_t j = j0 + lane;
                        bool ok = false;
                        uint32_t pos = kEmpty;
                        if (j < total) {
                            pos = G[j];
                            if (pos != kEmpty) ok = hash_insert(H, A.hs, A.hshift, pos);
                        }
                        append(w.P(A), nb, ok, pos);
                    }
                }
                __syncwarp();
            }
            hcount += nb;
            if (nb == 0) continue;
            const uint32_t ns = eval_sort<NCH, BYTES>(A, w.base, nb, w.T(A)[A.L - 1], 0);
            st_dist += nb;
            merge_step(A, w, A.L, 0, ns, false);
        }
        // post-filter: the in-range entries of the final list, in order
        {
            const key_t* T = w.T(A);
            key_t* Tn = w.Tn(A);
            uint32_t nin = 0;
            for (uint32_t i0 = 0; i0 < A.L; i0 += 32) {
                const uint32_t i = i0 + lane;
                const key_t k = i < A.L ? T[i] : kEmptyKey;
                const bool ok = k != kEmptyKey && (k & kKeyInRange);
                const uint32_t msk = __ballot_sync(kFull, ok);
                if (ok) Tn[nin + __popc(msk & lanemask_lt())] = k;
                nin += __popc(msk);
            }
            __syncwarp();
            write_result(A, q, Tn, nin);
        }
        __syncwarp();
        if (lane == 0) {
            atomicAdd(A.stats + 0, (unsigned long long)st_dist);
            atomicAdd(A.stats + 1, (unsigned long long)st_exp);
            atomicAdd(A.stats + 5, 1ull);
        }
    }
}

// Assembled graph of the full-graph search (assemble_edges, full_graph_search.cuh:984-997):
// row of position p, slot j * reserve + e: in p's own cell the e-th entry of its graph row,
// in every other cell j its e-th cross edge (positions; kEmpty where absent).
__global__ void assemble_kernel(const uint32_t* __restrict__ graph, const uint32_t* __restrict__ cross,
                                const uint32_t* __restrict__ spk, const uint32_t* __restrict__ seg, uint32_t n,
                                uint32_t P, uint32_t R, uint32_t E, uint32_t reserve, uint32_t* __restrict__ out) {
    const uint64_t D = (uint64_t)P * reserve, total = (uint64_t)n * D;
    for (uint64_t idx = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; idx < total;
         idx += (uint64_t)gridDim.x * blockDim.x) {
        const uint32_t pos = (uint32_t)(idx / D), slot = (uint32_t)(idx % D), j = slot / reserve, e = slot % reserve;
        uint32_t lo = 0, hi = P;  // seg[lo] <= pos < seg[hi]: the own cell
        while (hi - lo > 1) {
            const uint32_t mid = (lo + hi) >> 1;
            if (seg[mid] <= pos)
                lo = mid;
            else
                hi = mid;
        }
        uint32_t v = kEmpty;
        if (j == lo) {
            if (e < R) v = graph[(size_t)pos * R + e];
        } else if (e < E && cross) {
            const uint32_t row = spk ? spk[pos] : pos;
            v = cross[(size_t)row * P * E + (size_t)j * E + e];
        }
        out[idx] = v;
    }
}

__global__ void run_to_ids_kernel(const unsigned long long* __restrict__ run, uint32_t total,
                                  const uint32_t* __restrict__ i2g, uint32_t* ids, float* dist) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= total) return;
    const key_t k = run[i];
    if (ids) ids[i] = k == kEmptyKey ? kEmpty : i2g[key_pos(k)];
    if (dist) dist[i] = k == kEmptyKey ? kInf : key_dist(k);
}

// k-way merge of per-shard result keys: keys[(g * qnum + q) * k + i], each list sorted and
// the lists disjoint; one warp per query ranks every key against all lists.
__global__ void merge_lists_kernel(const unsigned long long* __restrict__ keys, uint32_t lists, uint32_t qnum,
                                   uint32_t k, const uint32_t* __restrict__ i2g, uint32_t* ids, float* dist) {
    const uint32_t q = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (q >= qnum) return;
    const uint32_t lane = lane_id();
    for (uint32_t i = lane; i < k; i += 32) {
        ids[(size_t)q * k + i] = kEmpty;
        if (dist) dist[(size_t)q * k + i] = kInf;
    }
    __syncwarp();
    for (uint32_t j = lane; j < lists * k; j += 32) {
        const uint32_t g = j / k, i = j - g * k;
        const key_t x = keys[((size_t)g * qnum + q) * k + i];
        if (x == kEmptyKey) continue;
        uint32_t rank = i;
        for (uint32_t h = 0; h < lists && rank < k; ++h)
            if (h != g) rank += keys_below(keys + ((size_t)h * qnum + q) * k, k, x);
        if (rank < k) {
            ids[(size_t)q * k + rank] = i2g[key_pos(x)];
            if (dist) dist[(size_t)q * k + rank] = key_dist(x);
        }
    }
}

typedef void (*KernelFn)(const SArgs);

// Row lengths compiled with a fixed chunk count (fp16: d8 / 8, bytes: d16 / 16); others
// use the generic kernel.
KernelFn pick_kernel(uint32_t nch, bool bytes) {
    if (bytes) {
        switch (nch) {
            case 8: return gmg_search_kernel<8, true>;
            default: return gmg_search_kernel<0, true>;
        }
    }
    switch (nch) {
        case 4: return gmg_search_kernel<4, false>;
        case 8: return gmg_search_kernel<8, false>;
        case 12: return gmg_search_kernel<12, false>;
        case 16: return gmg_search_kernel<16, false>;
        case 32: return gmg_search_kernel<32, false>;
        case 96: return gmg_search_kernel<96, false>;
        default: return gmg_search_kernel<0, false>;
    }
}

KernelFn pick_fullgraph(uint32_t nch, bool bytes) {
    if (bytes) return nch == 8 ? fullgraph_kernel<8, true> : fullgraph_kernel<0, true>;
    switch (nch) {
        case 16: return fullgraph_kernel<16, false>;
        case 8: return fullgraph_kernel<8, false>;
        default: return fullgraph_kernel<0, false>;
    }
}

}  // namespace

CellView shard_view(const DeviceIndex& d) {
    CellView v;
    v.slot = d.sh_slot;
    v.gofs = d.sh_gofs;
    v.xofs = d.sh_xofs;
    v.vsh = d.sh_vsh;
    v.graph = d.graph;
    v.cross = d.cross;
    v.nslots = (uint32_t)d.shard_cells.size();
    v.xstride = d.E;
    return v;
}

namespace {
// Queries of a whole-index search that take the exact route (the search kernel's rule:
// a non-empty cell list and >= postfilter cells or a box share <= prefilter; with route_slots
// > 0 also a box count below route_slots x cells, the cost rule of gf_search_params.route)
// are marked for the tensor-core exact scan (gf_search_params.exact_tc); their number goes
// to n_exact and n_queries.
__global__ void mark_exact_kernel(const uint32_t* __restrict__ counts, const uint32_t* __restrict__ box, uint32_t n,
                                  uint32_t qnum, uint32_t postfilter, float prefilter, unsigned long long route_slots,
                                  uint32_t* __restrict__ mark, unsigned long long* stats) {
    const uint32_t q = blockIdx.x * blockDim.x + threadIdx.x;
    bool ex = false;
    if (q < qnum) {
        const uint32_t nc = counts[q];
        ex = nc > 0 && (nc >= postfilter || (box && (float)((double)box[q] / (double)n) <= prefilter) ||
                        (box && route_slots && (unsigned long long)box[q] < route_slots * nc));
        mark[q] = ex ? 1u : 0u;
    }
    const uint32_t b = __ballot_sync(kFull, ex);
    if (lane_id() == 0 && b) {
        atomicAdd(stats + 4, (unsigned long long)__popc(b));  // n_exact
        atomicAdd(stats + 5, (unsigned long long)__popc(b));  // n_queries (the search kernel skips them)
    }
}
}  // namespace

gf_status search(gf_index* idx, gf_plan* plan, const gf_search_params* prm, uint32_t* ids, float* dist,
                 cudaStream_t s, const CellView* view, bool fullgraph) {
    DeviceIndex& d = idx->d;
    Plan& p = plan->p;
    if (!p.planned) return fail(GF_ERR_STATE, "gf_search before gf_plan_queries");
    if (fullgraph && (view || !d.fgraph))
        return fail(GF_ERR_STATE, "full-graph search needs the assembled graph (gf_index_assemble)");
    gf_search_params P;
    gf_search_defaults(&P);
    if (prm) P = *prm;
    if (P.k == 0 || P.k > 1024) return fail(GF_ERR_ARG, "k must be 1..1024");
    if (P.L < P.k || P.L > 4096) return fail(GF_ERR_ARG, "L must be k..4096");
    if (P.width == 0 || P.width > 32) return fail(GF_ERR_ARG, "width must be 1..32");
    if (P.route > 1) return fail(GF_ERR_ARG, "route must be 0 or 1");
    if (P.route && !P.exact_tc) return fail(GF_ERR_ARG, "route = 1 sends queries to the tensor-core exact scan: set exact_tc");
    if (P.route && !(p.prefilter > 0.0f) && !d.at_ok)
        return fail(GF_ERR_STATE, "route = 1 needs box counts: an index with attribute tiles, or a plan built with "
                                  "prefilter > 0");
    if (P.exact_tc) {
        if (view || fullgraph || d.sharded || d.host_graph)
            return fail(GF_ERR_ARG, "exact_tc applies to gf_search / gf_search_host on a whole device-resident index");
        if (!bf_tc_usable(d, P.k))
            return fail(GF_ERR_STATE, "exact_tc needs an index with keep_fp32 rows (dim <= 1024, finite) and k <= 128");
    }
    uint32_t n_entry = P.n_entry ? P.n_entry : d.degree;
    n_entry = std::min<uint32_t>(n_entry, fullgraph ? d.fentry_n : (uint32_t)d.entry_h.size());
    if (!ids && !(view && view->run)) return fail(GF_ERR_ARG, "null ids_out");
    if (!view && d.sharded && !fullgraph) {
        // a shard: search its cells through its view, merge into the plan's running keys
        const size_t need = (size_t)p.qnum * P.k;
        if (need > p.run_cap) {
            GF_CUDA(cudaStreamSynchronize(s));
            if (p.run) cudaFree(p.run);
            p.run = nullptr;
            p.run_cap = 0;
            GF_CUDA(cudaMalloc((void**)&p.run, std::max<size_t>(need, 1) * 8));
            p.run_cap = need;
        }
        CellView v = shard_view(d);
        v.run = p.run;
        GF_CUDA(cudaMemsetAsync(p.run, 0xFF, need * 8, s));
        gf_status st = search(idx, plan, &P, nullptr, nullptr, s, &v);
        if (st != GF_OK) return st;
        return finish_run(idx, p.run, (uint32_t)need, ids, dist, s);
    }
    if (!view && d.host_graph)
        return fail(GF_ERR_STATE, "the index keeps its graphs in host memory: search it with gf_search_batched");
    if (p.qnum == 0) return GF_OK;

    SArgs A;
    const bool bytes = d.codec != 0;
    A.vec16 = bytes ? d.vec8 : d.vec16;
    A.q32 = p.q32;
    A.csc = d.csc;
    A.cbi = d.cbi;
    A.alpha = d.alpha;
    A.xmask = d.codec == 1 ? 0x80808080u : 0u;
    A.dim = d.dim;
    A.attrs = d.attrs;
    A.graph = view ? view->graph : d.graph;
    A.cross = view ? view->cross : d.cross;
    A.slot = view ? view->slot : nullptr;
    A.gofs = view ? view->gofs : nullptr;
    A.xofs = view ? view->xofs : nullptr;
    A.vsh = view ? view->vsh : nullptr;
    A.run = view ? view->run : nullptr;
    A.nslots = view ? view->nslots : 0;
    A.xstride = view ? view->xstride : 0;
    A.seg = d.seg;
    A.i2g = d.i2g;
    A.spk = d.spk_rank;
    A.q16 = p.q16;
    A.lb = p.lb;
    A.rb = p.rb;
    A.counts = p.counts;
    A.offsets = p.offsets;
    A.cells = p.cells;
    A.box = p.prefilter > 0.0f ? p.box : nullptr;
    A.task = p.task;
    A.entry = fullgraph ? d.fentry : d.entry;
    A.queue = p.scratch;
    A.out_ids = ids;
    A.out_d = dist;
    A.stats = p.stats;
    A.qnum = p.qnum;
    A.nch = bytes ? d.d16 / 16 : d.d8 / 8;
    A.a = d.a;
    A.P = d.ncells;
    A.R = d.degree;
    A.E = (d.cross || d.cross_h) ? d.E : 0;
    A.L = P.L;
    A.K = P.k;
    A.W = P.width;
    A.max_iter = P.max_iter;
    A.n_entry = n_entry;
    A.postfilter = P.postfilter;
    A.n = d.n;
    A.prefilter = p.prefilter;
    A.wait_polls = P.test_wait ? P.test_wait : kStageWaitPolls;
    A.extra_tx = P.test_wait ? 16u : 0u;
    if (fullgraph) {  // one graph over the whole index: the assembled rows, no cross edges
        A.graph = d.fgraph;
        A.R = d.fdeg;
        A.cross = nullptr;
        A.E = 0;
        A.spk = nullptr;
    }
    A.graph_bulk = (A.R * 4) % 16 == 0 ? 1u : 0u;
    uint32_t need = std::max<uint32_t>({P.width * A.R, n_entry, kHopSlots * A.E, 64u});
    uint32_t bcap = 1;
    while (bcap < need) bcap <<= 1;
    A.bcap = bcap;
    uint32_t hs = P.hash_slots;
    if (hs == 0) {
        hs = 256;
        while (hs < 2 * (P.L + bcap)) hs <<= 1;
    }
    if (hs & (hs - 1)) return fail(GF_ERR_ARG, "hash_slots must be a power of two");
    if (hs < 2 * (P.L + bcap)) return fail(GF_ERR_ARG, "hash_slots below 2*(L + batch)");
    A.hs = hs;
    uint32_t lg = 0;
    while ((1u << lg) < hs) ++lg;
    A.hshift = 32 - lg;
    // staging: up to 16 rows of an odd number of 16-byte chunks, at most 4.5 KB per warp; rows
    // of 1 KB and more get up to 12.5 KB, so that a copy round still brings 8 rows (with 4.5 KB
    // a 768-dim fp16 row allowed 2, leaving 28 of 32 lanes idle and the copy latency exposed
    // once per 2 rows)
    const uint32_t nch16 = (A.nch + 15) / 16 * 16;
    A.stage_stride = A.nch | 1u;
    const uint32_t stage_budget = A.nch >= 64 ? 12800u : 4608u;
    uint32_t sr = 16;
    while (sr > 1 && sr * A.stage_stride * 16 > stage_budget) sr >>= 1;
    A.stage_rows = sr;
    A.stage_shift = 0;
    while ((1u << A.stage_shift) < sr) ++A.stage_shift;
    // exact for the hop's j < 64 E, E <= 4 (j * (e_magic * E - 2^32) < 2^32)
    A.e_magic = A.E ? ((1ull << 32) + A.E - 1) / A.E : 0ull;
    make_layout(A, nch16, bytes);

    KernelFn kern = fullgraph ? pick_fullgraph(A.nch, bytes) : pick_kernel(A.nch, bytes);
    const int warps_per_block = 4;
    size_t smem = (size_t)warps_per_block * A.warp_words * 4;
    int dev = d.device;
    int max_optin = 0, nsm = 0;
    cudaDeviceGetAttribute(&max_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
    if (smem > (size_t)max_optin) return fail(GF_ERR_ARG, "L/k/hash too large for shared memory");
    GF_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    int per_sm = 0;
    GF_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, 128, smem));
    if (per_sm < 1) return fail(GF_ERR_ARG, "search kernel does not fit on an SM");
    uint32_t blocks = (uint32_t)(nsm * per_sm);
    uint32_t need_blocks = (p.qnum + warps_per_block - 1) / warps_per_block;
    blocks = std::min(blocks, need_blocks);
    GF_CUDA(cudaMemsetAsync(p.scratch, 0, sizeof(uint32_t), s));
    if (!(view && view->accumulate_stats)) GF_CUDA(cudaMemsetAsync(p.stats, 0, 8 * sizeof(unsigned long long), s));
    if (!view && !fullgraph && d.at_ok && d.cells_hold_rows) {  // exact route through the attribute tiles
        A.sbox = d.bf_sbox;
        A.tbox = d.bf_tbox;
        A.tattrs = d.bf_attrs;
        A.trow = d.bf_rowpos;
        A.nstiles = d.bf_stiles;
        A.ntiles = d.bf_tiles;
        A.a8 = (d.a + 3) & ~3u;
    }
    if (P.exact_tc) {
        // exact-route queries: the tensor-core exact scan writes their rows, the search kernel
        // skips them
        if (!p.xmark) GF_CUDA(cudaMalloc((void**)&p.xmark, sizeof(uint32_t) * std::max<uint32_t>(p.max_q, 1)));
        const unsigned long long route_slots =
            P.route ? (unsigned long long)GF_ROUTE_ROWS_PER_SLOT * (P.L + kHopSlots) : 0ull;
        const uint32_t* box = A.box;
        if (P.route && !box) {
            // no exact counts in the plan: the cost rule takes the tile-level estimate
            box_count_tiles(d, p.lb, p.rb, p.qnum, p.box, s, true);
            box = p.box;
        }
        mark_exact_kernel<<<(p.qnum + 255) / 256, 256, 0, s>>>(p.counts, box, d.n, p.qnum, P.postfilter,
                                                                A.box ? p.prefilter : 0.0f, route_slots, p.xmark,
                                                                p.stats);
        GF_CUDA(cudaGetLastError());
        gf_status st = bruteforce(idx, p.q32, p.lb, p.rb, p.qnum, P.k, ids, dist, s, nullptr, p.xmark);
        if (st != GF_OK) return st;
        A.skip = p.xmark;
    }
    kern<<<blocks, 128, smem, s>>>(A);
    GF_CUDA(cudaGetLastError());
    return GF_OK;
}

gf_status finish_run(gf_index* idx, const unsigned long long* run, uint32_t total, uint32_t* ids, float* dist,
                     cudaStream_t s) {
    if (total == 0) return GF_OK;
    run_to_ids_kernel<<<(total + 255) / 256, 256, 0, s>>>(run, total, idx->d.i2g, ids, dist);
    GF_CUDA(cudaGetLastError());
    return GF_OK;
}

}  // namespace gf

using namespace gf;

extern "C" gf_status gf_index_assemble(gf_index* idx, uint32_t reserve) {
    if (!idx) return fail(GF_ERR_ARG, "null index");
    DeviceIndex& d = idx->d;
    if (d.sharded || d.host_graph) return fail(GF_ERR_STATE, "the assembled graph needs a whole device-resident index");
    if (reserve == 0 || reserve > 16) return fail(GF_ERR_ARG, "reserve must be 1..16");
    if ((uint64_t)d.ncells * reserve > 4096) return fail(GF_ERR_ARG, "cells x reserve above 4096");
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(d.device);
    gf_status st = GF_OK;
    do {
        if (d.fgraph) {
            cudaFree(d.fgraph);
            d.fgraph = nullptr;
        }
        const uint32_t D = d.ncells * reserve;
        cudaError_t e = cudaMalloc((void**)&d.fgraph, std::max<size_t>((size_t)d.n * D, 1) * 4);
        if (e != cudaSuccess) {
            st = cuda_fail(e, "assembled graph");
            break;
        }
        assemble_kernel<<<148 * 8, 256>>>(d.graph, d.cross, d.spk_rank, d.seg, d.n, d.ncells, d.degree, d.E,
                                          reserve, d.fgraph);
        // entry positions over the whole index: std::mt19937 default seed, draw % n, distinct
        std::mt19937 rng;
        std::vector<uint32_t> ent;
        const uint32_t want = std::min<uint32_t>(std::max<uint32_t>(D, 64), d.n);
        std::vector<uint8_t> seen(d.n, 0);
        while (ent.size() < want) {
            const uint32_t t = (uint32_t)(rng() % d.n);
            if (!seen[t]) {
                seen[t] = 1;
                ent.push_back(t);
            }
        }
        if (d.fentry) cudaFree(d.fentry);
        d.fentry = nullptr;
        e = cudaMalloc((void**)&d.fentry, std::max<size_t>(ent.size(), 1) * 4);
        if (e == cudaSuccess) e = cudaMemcpy(d.fentry, ent.data(), ent.size() * 4, cudaMemcpyHostToDevice);
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
        if (e != cudaSuccess) {
            st = cuda_fail(e, "assembled graph");
            break;
        }
        d.fdeg = D;
        d.fentry_n = (uint32_t)ent.size();
        d.fentry_h = ent;
    } while (0);
    if (prev >= 0) cudaSetDevice(prev);
    return st;
}

extern "C" gf_status gf_search_fullgraph(gf_index* idx, gf_plan* plan, const gf_search_params* params,
                                         uint32_t* ids_out, float* dist_out, void* stream) {
    if (!idx || !plan || plan->p.idx != idx) return fail(GF_ERR_ARG, "plan does not belong to this index");
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(idx->d.device);
    gf_status st = search(idx, plan, params, ids_out, dist_out, (cudaStream_t)stream, nullptr, true);
    if (prev >= 0) cudaSetDevice(prev);
    return st;
}

extern "C" gf_status gf_search_keys(gf_index* idx, gf_plan* plan, const gf_search_params* params, uint64_t* keys_out,
                                    void* stream) {
    if (!idx || !plan || plan->p.idx != idx) return fail(GF_ERR_ARG, "plan does not belong to this index");
    if (!keys_out) return fail(GF_ERR_ARG, "null keys_out");
    DeviceIndex& d = idx->d;
    if (d.host_graph) return fail(GF_ERR_STATE, "the index keeps its graphs in host memory");
    if (!plan->p.planned) return fail(GF_ERR_STATE, "gf_search_keys before gf_plan_queries");
    gf_search_params P;
    gf_search_defaults(&P);
    if (params) P = *params;
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(d.device);
    CellView v;
    if (d.sharded) {
        v = shard_view(d);
    } else {
        v.graph = d.graph;
        v.cross = d.cross;
    }
    v.run = reinterpret_cast<unsigned long long*>(keys_out);
    const cudaStream_t s = (cudaStream_t)stream;
    gf_status st = GF_OK;
    cudaError_t e = cudaMemsetAsync(keys_out, 0xFF, (size_t)plan->p.qnum * P.k * 8, s);
    if (e != cudaSuccess)
        st = cuda_fail(e, "gf_search_keys");
    else
        st = gf::search(idx, plan, &P, nullptr, nullptr, s, &v);
    if (prev >= 0) cudaSetDevice(prev);
    return st;
}

extern "C" gf_status gf_merge_keys(gf_index* idx, const uint64_t* keys, uint32_t n_lists, uint32_t qnum, uint32_t k,
                                   uint32_t* ids_out, float* dist_out, void* stream) {
    if (!idx) return fail(GF_ERR_ARG, "null index");
    if (qnum == 0) return GF_OK;
    if (!keys || !ids_out || n_lists == 0 || k == 0) return fail(GF_ERR_ARG, "null argument or zero size");
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(idx->d.device);
    const uint32_t warps = 4;
    merge_lists_kernel<<<(qnum + warps - 1) / warps, 32 * warps, 0, (cudaStream_t)stream>>>(
        reinterpret_cast<const unsigned long long*>(keys), n_lists, qnum, k, idx->d.i2g, ids_out, dist_out);
    cudaError_t e = cudaGetLastError();
    if (prev >= 0) cudaSetDevice(prev);
    if (e != cudaSuccess) return cuda_fail(e, "gf_merge_keys");
    return GF_OK;
}
