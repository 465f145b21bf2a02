// Exact filtered k-NN (gf_bruteforce) with the query x point products on the tensor cores.
// Replaces the fp16 distance scan of prefiltering_and_bruteforce / dis_cal_reduce
// (brute_force.cuh:252-405) and gives the same answer as naive_brute_force_with_filter
// (gpu_graph.cu:10782-10812) restated with the canonical fp32 distance.
//
// Index side (bf_tc_prepare, once per index that keeps fp32 rows): the rows are centred on
// their mean m, scaled by a power of two s so that |s (x - m)| < 2^14, and rounded to fp16.
// The copy X~ is stored pre-tiled, 128 points per tile, in the tcgen05 K-major no-swizzle
// layout (8 rows x 16 bytes per core matrix; 64-element chunks of 8 core-matrix columns),
// so one bulk copy per chunk fills a shared-memory stage.  Per point: px = (1 - kappa)|x~|^2
// rounded down and the rounding residual delta_x = |x - (m + x~ / s)| rounded up; per tile:
// the bounding box of its points' attributes.
//
// Query side (one gf_bruteforce call):
//  1. queries are ordered by the Morton code of their box centre, so that 128 consecutive
//     queries (one tile) and 32 (one epilogue warp) ask for nearby boxes;
//  2. bf_prep_kernel writes q~ = fp16(s (q - m)) in the same tiled layout, pq and delta_q;
//  3. bf_boxes_kernel / bf_tiles_kernel: per query tile the union of its boxes and the list
//     of point tiles whose attribute bounds meet it (other tiles cannot hold an answer);
//  4. bf_tc_kernel, per (query tile, share of its point tiles): one thread issues bulk
//     copies of the point chunks into a ring of shared-memory stages and the tcgen05.mma
//     (kind::f16, M = N = 128, fp32 accumulation) of each tile into one of four TMEM
//     accumulators; eight epilogue warps read the accumulators (tcgen05.ld, one query per
//     TMEM lane, two warps per lane quarter taking alternate tiles) and form
//     a = px - 2 S; a thread keeps its query's KM smallest a among in-box points (a heap in
//     shared memory; KM = 32 for k <= 16, 128 with one warp per lane quarter for k <= 128)
//     -- a point is tested against the box only when a is below the list's current KM-th
//     value, which after the first few tiles is rare;
//  5. bf_merge_kernel (a warp per query): merges the lists, re-ranks the KM smallest a with
//     the canonical fp32 distance (dist32, oracle orc_dist32) and proves the result: every
//     point left out has a >= a*, hence a canonical distance >= LB(a*) (the error bound
//     below); when LB(a*) is not above the k-th re-ranked distance, or the query could not
//     be handled here, the query goes to a list that the CUDA-core kernel
//     (bruteforce_kernel) answers afterwards.  The result is the canonical one in every case.
//
// Error bound.  With T = |q~|^2 + |x~|^2 - 2 q~.x~ (exact), the tensor cores return S with
// 2|S - q~.x~| <= kappa (|q~|^2 + |x~|^2), kappa = (2 Dp + 64) 2^-23 (products of fp16 values
// are exact in fp32; the fp32 accumulation of Dp products with truncation errs by at most
// Dp 2^-23 sum|q~_i x~_i| <= Dp 2^-23 |q~||x~|; the bound doubles that and adds 64 units).
// So T >= pq + a, and a point with fl(a) >= a* has T >= pq + a* - 2^-22 |a*|.  Then
// |q - x| >= sqrt(T) / s - delta_q - delta_max, and the canonical fp32 sum of D squared
// differences is >= |q - x|^2 (1 - eta), eta = (D/8 + 16) 2^-23.
#include <cub/cub.cuh>

#include <algorithm>
#include <cmath>
#include <cstring>

#include "gf_device.cuh"
#include "gf_internal.h"

namespace gf {
namespace {

using namespace dev;

constexpr uint32_t kBM = 128;          // queries per tile (TMEM lanes)
constexpr uint32_t kBN = kTileRows;    // points per tile (accumulator columns)
constexpr uint32_t kKC = 64;           // elements per K chunk of the index layout (8 core-matrix columns)
constexpr uint32_t kChunkBytes = kBN * kKC * 2;  // 16 KB
// The tiled layouts are column-major over 8-element core-matrix columns, so elements
// [e, e + m) of a 128-row tile (e, m multiples of 16) are one contiguous run of m * 256 bytes
// starting at half e * 128: a pipeline stage can carry any multiple of 16 elements.  A call
// stages kc = 64 or 32 elements at a time (TcArgs::kc), whichever keeps more bytes in flight.
constexpr uint32_t kColBytes = kBN * 16;         // one 16-byte core-matrix column of 128 rows
constexpr uint32_t kAcc = 4;           // TMEM accumulators of kBN columns
constexpr uint32_t kMeta = 8;          // tile metadata slots (copies run up to kMeta tiles ahead)
constexpr uint32_t kSlots = 16;        // CTAs that may share one query tile
// Candidate lists of one query row.  Shallow (k <= 16): 32 entries; two epilogue warps per
// TMEM lane quarter take alternate tiles (8 epilogue warps, 2 lists per query and CTA).
// Deep (16 < k <= 128): 128 entries; one warp per lane quarter takes every tile (4 epilogue
// warps, 1 list per query and CTA), so that the lists still fit in shared memory.
template <bool DEEP>
struct Lists {
    static constexpr uint32_t KM = DEEP ? 128 : 32;   // candidates kept per list
    static constexpr uint32_t NPAR = DEEP ? 1 : 2;    // tile parities
    static constexpr uint32_t EW = 4 * NPAR;          // epilogue warps
    static constexpr uint32_t OWN = 32 * EW;          // list owners (epilogue threads)
    static constexpr uint32_t THREADS = 64 + OWN;     // producer warp, MMA warp, epilogue warps
    static constexpr uint32_t LISTS = kSlots * NPAR;  // lists per query, merged by one warp
};
constexpr uint32_t kMaxKShallow = 16;
constexpr uint32_t kMaxDp = 1024;
constexpr uint32_t kResidentDp = 256;  // query tiles up to this width stay in shared memory
constexpr uint32_t kMaxK = 128;
constexpr uint32_t kPolls = 1u << 20;
constexpr uint32_t kSmemLimit = 227 * 1024;

// Instruction descriptor, kind::f16: D f32, A and B f16, both K-major, N = kBN, M = kBM.
constexpr uint32_t kIdesc = (1u << 4) | ((kBN >> 3) << 17) | ((kBM >> 4) << 24);

__device__ __forceinline__ uint64_t kmajor_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;
    return d;
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void mma_f16(uint32_t tmem, uint64_t ad, uint64_t bd, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem),
        "l"(ad), "l"(bd), "r"(kIdesc), "r"(acc), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// 32 consecutive TMEM columns of this warp's 32 lanes (lane i gets row i).
__device__ __forceinline__ void tmem_ld32(uint32_t addr, uint32_t* v) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
          "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
          "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
          "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(addr));
}
// Wait for this thread's tcgen05.ld; names the 32 registers of an earlier tcgen05.ld as operands so that no use of
// them is scheduled before it.
__device__ __forceinline__ void tmem_wait_ld(uint32_t* v) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]), "+r"(v[6]), "+r"(v[7]),
                   "+r"(v[8]), "+r"(v[9]), "+r"(v[10]), "+r"(v[11]), "+r"(v[12]), "+r"(v[13]), "+r"(v[14]),
                   "+r"(v[15]), "+r"(v[16]), "+r"(v[17]), "+r"(v[18]), "+r"(v[19]), "+r"(v[20]), "+r"(v[21]),
                   "+r"(v[22]), "+r"(v[23]), "+r"(v[24]), "+r"(v[25]), "+r"(v[26]), "+r"(v[27]), "+r"(v[28]),
                   "+r"(v[29]), "+r"(v[30]), "+r"(v[31])
                 :
                 : "memory");
}

// Bounded wait on a phase (at most `polls` polls); false when it ran out or the CTA is stopping.
__device__ __forceinline__ bool bwait(uint64_t* bar, uint32_t par, const volatile uint32_t* stop, uint32_t polls) {
    for (uint32_t p = 0; p < polls; ++p) {
        if (mbar_try_wait(bar, par, 1000)) return true;
        if (*stop) return false;
    }
    return false;
}

// Half index of element i of row `row` in a 128-row tile (core-matrix layout, 64-element
// chunks): chunk i/64, 16-byte column (i%64)/8, 8-row group row/8.
__device__ __forceinline__ size_t cm_half(uint32_t row, uint32_t i) {
    return (size_t)(i >> 6) * (kBN * kKC) + ((i & 63u) >> 3) * (kBN * 8) + (row >> 3) * 64 + (row & 7u) * 8 + (i & 7u);
}

__device__ __forceinline__ uint32_t f2ord(float f) {
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float ord2f(uint32_t o) {
    return __uint_as_float((o & 0x80000000u) ? (o & 0x7FFFFFFFu) : ~o);
}

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
    return v;
}

// ------------------------------------------------------------------ index preparation

// Morton code of an attribute vector (a <= 8 attributes, 63 / a bits each, at most 21),
// each attribute normalised by the index's attribute range (origin alo, 1 / extent ainv).
__device__ __forceinline__ uint64_t attr_morton(const float* v, uint32_t a, const float* __restrict__ alo,
                                                const float* __restrict__ ainv) {
    const uint32_t bits = min(21u, 63u / a);
    uint64_t code = 0;
    for (uint32_t j = 0; j < a; ++j) {
        float t = (v[j] - alo[j]) * ainv[j];
        t = isfinite(t) ? fminf(fmaxf(t, 0.0f), 1.0f) : 0.0f;
        const uint32_t q = min((uint32_t)(t * (float)(1u << bits)), (1u << bits) - 1u);
        for (uint32_t b = 0; b < bits; ++b) code |= (uint64_t)((q >> b) & 1u) << (b * a + j);
    }
    return code;
}

// Sort keys of the points for the tensor-core copy: Morton order of their attributes, so that
// a 128-point tile covers a small region of attribute space.
__global__ void bf_point_keys_kernel(const float* __restrict__ attrs, uint32_t n, uint32_t a,
                                     const float* __restrict__ alo, const float* __restrict__ ainv,
                                     unsigned long long* __restrict__ keys, uint32_t* __restrict__ vals) {
    const uint32_t p = blockIdx.x * blockDim.x + threadIdx.x;
    if (p >= n) return;
    float v[kMaxAttr];
    for (uint32_t j = 0; j < a; ++j) v[j] = attrs[(size_t)p * a + j];
    keys[p] = attr_morton(v, a, alo, ainv);
    vals[p] = p;
}

// Column sums of the fp32 rows (double), for the mean.
__global__ void bf_colsum_kernel(const float* __restrict__ x, uint32_t n, uint32_t d4, uint32_t dim, double* sum) {
    const uint32_t per = (n + gridDim.x - 1) / gridDim.x;
    const uint32_t r0 = blockIdx.x * per, r1 = min(n, r0 + per);
    for (uint32_t c = threadIdx.x; c < dim; c += blockDim.x) {
        double s = 0.0;
        for (uint32_t r = r0; r < r1; ++r) s += (double)x[(size_t)r * d4 + c];
        atomicAdd(sum + c, s);
    }
}

// max |fl(x - m)| over all elements (float bits, non-negative) and a flag for non-finite values.
__global__ void bf_maxabs_kernel(const float* __restrict__ x, uint32_t n, uint32_t d4, uint32_t dim,
                                 const float* __restrict__ m, uint32_t* maxbits, uint32_t* bad) {
    uint32_t mx = 0, b = 0;
    const size_t total = (size_t)n * dim;
    for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < total; e += (size_t)gridDim.x * blockDim.x) {
        const uint32_t r = (uint32_t)(e / dim), c = (uint32_t)(e % dim);
        const float v = x[(size_t)r * d4 + c];
        if (!isfinite(v)) b = 1;
        const float dv = fabsf(__fsub_rn(v, m[c]));
        if (isfinite(dv)) mx = max(mx, __float_as_uint(dv));
    }
    for (int o = 16; o > 0; o >>= 1) {
        mx = max(mx, __shfl_xor_sync(kFull, mx, o));
        b |= __shfl_xor_sync(kFull, b, o);
    }
    if ((threadIdx.x & 31u) == 0) {
        atomicMax(maxbits, mx);
        if (b) atomicOr(bad, 1u);
    }
}

// One warp per point position (padding positions up to tiles*128 included): the tiled fp16
// copy, px and the residual norm; the largest residual is collected in dmax (float bits).
__global__ void bf_convert_kernel(const float* __restrict__ x, uint32_t n, uint32_t d4, uint32_t dim, uint32_t dp,
                                  const float* __restrict__ m, float s, double one_minus_kappa, uint32_t npad,
                                  const uint32_t* __restrict__ order, __half* __restrict__ xt, float* __restrict__ px,
                                  uint32_t* dmax) {
    const uint32_t lane = lane_id();
    const uint32_t warps = gridDim.x * (blockDim.x >> 5);
    for (uint32_t p = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); p < npad; p += warps) {
        __half* tile = xt + (size_t)(p / kBN) * kBN * dp;
        const uint32_t row = p % kBN;
        const uint32_t src = p < n ? order[p] : 0u;  // position of the point in row p
        double nx = 0.0, d2 = 0.0;
        for (uint32_t i = lane; i < dp; i += 32) {
            __half h = __float2half_rn(0.0f);
            if (p < n && i < dim) {
                const float v = x[(size_t)src * d4 + i];
                h = __float2half_rn(__fsub_rn(v, m[i]) * s);
                const double hv = (double)__half2float(h);
                nx += hv * hv;
                const double r = (double)v - (double)m[i] - hv / (double)s;
                d2 += r * r;
            }
            tile[cm_half(row, i)] = h;
        }
        nx = warp_sum_d(nx);
        d2 = warp_sum_d(d2);
        if (lane == 0) {
            if (p < n) {
                px[p] = __double2float_rd(one_minus_kappa * nx);
                const float dl = __double2float_ru(sqrt(d2) * (1.0 + 1e-12));
                atomicMax(dmax, __float_as_uint(dl));
            } else {
                px[p] = __int_as_float(0x7f800000);
            }
        }
    }
}

// Attribute bounds of each 128-point tile, tbox[t] = lo[a8], hi[a8] (one warp per tile; an
// empty tile gets lo > hi; unused entries lo = -inf, hi = +inf), and the tile-padded attribute
// copy (NaN past n, so no padding point is ever inside a box).
__global__ void bf_tilebox_kernel(const float* __restrict__ attrs, uint32_t n, uint32_t a, uint32_t a8,
                                  uint32_t tiles, const uint32_t* order, float* __restrict__ tbox,
                                  float* __restrict__ pattrs, uint32_t* rowpos,  // order may alias rowpos
                                  uint32_t* __restrict__ tcnt) {
    const uint32_t lane = lane_id();
    const uint32_t t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (t >= tiles) return;
    {  // points of the tile whose attributes are all numbers (a NaN is inside no box)
        uint32_t c = 0;
        for (uint32_t r = lane; r < kBN; r += 32) {
            const uint32_t p = t * kBN + r;
            bool ok = p < n;
            for (uint32_t j = 0; ok && j < a; ++j) {
                const float v = attrs[(size_t)order[p] * a + j];
                ok = v == v;
            }
            c += ok;
        }
        for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(kFull, c, o);
        if (lane == 0) tcnt[t] = c;
    }
    for (uint32_t r = lane; r < kBN; r += 32) {
        const uint32_t p = t * kBN + r;
        rowpos[p] = p < n ? order[p] : kEmpty;
    }
    for (uint32_t j = 0; j < a8; ++j) {
        float lo = __int_as_float(0x7f800000), hi = -__int_as_float(0x7f800000);
        for (uint32_t r = lane; j < a && r < kBN; r += 32) {
            const uint32_t p = t * kBN + r;
            float v = __int_as_float(0x7fc00000);
            if (p < n) {
                v = attrs[(size_t)order[p] * a + j];
                lo = fminf(lo, v);
                hi = fmaxf(hi, v);
            }
            pattrs[(size_t)p * a + j] = v;
        }
        for (int o = 16; o > 0; o >>= 1) {
            lo = fminf(lo, __shfl_xor_sync(kFull, lo, o));
            hi = fmaxf(hi, __shfl_xor_sync(kFull, hi, o));
        }
        if (lane == 0) {
            tbox[(size_t)t * 2 * a8 + j] = j < a ? lo : -__int_as_float(0x7f800000);
            tbox[(size_t)t * 2 * a8 + a8 + j] = j < a ? hi : __int_as_float(0x7f800000);
        }
    }
}

// ------------------------------------------------------------------ per-call kernels

// Morton code of the box centre (the points' code of the same attribute space).
// Queries left out by the mask get the largest key: they sort behind every other query, so
// the trailing query tiles hold only them and meet no point tile.
__global__ void bf_morton_kernel(const float* __restrict__ lb, const float* __restrict__ rb, uint32_t qnum, uint32_t a,
                                 const float* __restrict__ alo, const float* __restrict__ ainv,
                                 const uint32_t* __restrict__ qmask, unsigned long long* keys, uint32_t* vals) {
    const uint32_t q = blockIdx.x * blockDim.x + threadIdx.x;
    if (q >= qnum) return;
    float c[kMaxAttr];
    for (uint32_t j = 0; j < a; ++j) c[j] = 0.5f * (lb[(size_t)q * a + j] + rb[(size_t)q * a + j]);
    keys[q] = (qmask && !qmask[q]) ? ~0ull : attr_morton(c, a, alo, ainv);
    vals[q] = q;
}

// One warp per sorted row r < qpad: the tiled fp16 query, pq, delta_q and the routing flag
// (1 = no query, 2 = the query cannot be handled on the tensor cores).
__global__ void bf_prep_kernel(const float* __restrict__ queries, uint32_t qnum, uint32_t dim, uint32_t dp,
                               const uint32_t* __restrict__ sorted, const uint32_t* __restrict__ qmask, uint32_t qpad,
                               const float* __restrict__ m, float s,
                               double one_minus_kappa, uint32_t* __restrict__ perm, __half* __restrict__ at,
                               float* __restrict__ pq, float* __restrict__ dq, uint32_t* __restrict__ flag,
                               uint32_t* __restrict__ thr_g) {
    const uint32_t lane = lane_id();
    const uint32_t r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (r >= qpad) return;
    uint32_t q = r < qnum ? sorted[r] : kEmpty;
    if (q != kEmpty && qmask && !qmask[q]) q = kEmpty;  // left out: a row without a query
    __half* tile = at + (size_t)(r / kBM) * kBM * dp;
    const uint32_t row = r % kBM;
    double nq = 0.0, d2 = 0.0;
    bool bad = false;
    for (uint32_t i = lane; i < dp; i += 32) {
        __half h = __float2half_rn(0.0f);
        if (q != kEmpty && i < dim) {
            const float v = queries[(size_t)q * dim + i];
            const float c = __fsub_rn(v, m[i]) * s;
            if (!(fabsf(c) <= 60000.0f)) {
                bad = true;
            } else {
                h = __float2half_rn(c);
                const double hv = (double)__half2float(h);
                nq += hv * hv;
                const double e = (double)v - (double)m[i] - hv / (double)s;
                d2 += e * e;
            }
        }
        tile[cm_half(row, i)] = h;
    }
    bad = __any_sync(kFull, bad);
    nq = warp_sum_d(nq);
    d2 = warp_sum_d(d2);
    if (lane == 0) {
        perm[r] = q;
        pq[r] = __double2float_rd(one_minus_kappa * nq);
        dq[r] = __double2float_ru(sqrt(d2) * (1.0 + 1e-12));
        flag[r] = q == kEmpty ? 1u : (bad ? 2u : 0u);
        thr_g[r] = f2ord(__int_as_float(0x7f800000));
    }
}

// Per query tile (128 threads, one per row): union of the rows' boxes, for the tile and
// for each group of 32 rows.  Rows without a query or with an empty box add nothing.
__global__ void bf_boxes_kernel(const float* __restrict__ lb, const float* __restrict__ rb, uint32_t a,
                                const uint32_t* __restrict__ perm, const uint32_t* __restrict__ flag,
                                float* __restrict__ tile_lo, float* __restrict__ tile_hi, float* __restrict__ grp_lo,
                                float* __restrict__ grp_hi) {
    __shared__ float wl[4][kMaxAttr], wh[4][kMaxAttr];
    const uint32_t r = blockIdx.x * kBM + threadIdx.x, lane = lane_id(), w = threadIdx.x >> 5;
    const uint32_t q = perm[r];
    bool use = flag[r] == 0;
    if (use)
        for (uint32_t j = 0; j < a; ++j) use = use && lb[(size_t)q * a + j] <= rb[(size_t)q * a + j];
    for (uint32_t j = 0; j < a; ++j) {
        float lo = use ? lb[(size_t)q * a + j] : __int_as_float(0x7f800000);
        float hi = use ? rb[(size_t)q * a + j] : -__int_as_float(0x7f800000);
        for (int o = 16; o > 0; o >>= 1) {
            lo = fminf(lo, __shfl_xor_sync(kFull, lo, o));
            hi = fmaxf(hi, __shfl_xor_sync(kFull, hi, o));
        }
        if (lane == 0) {
            wl[w][j] = lo;
            wh[w][j] = hi;
            grp_lo[((size_t)blockIdx.x * 4 + w) * a + j] = lo;
            grp_hi[((size_t)blockIdx.x * 4 + w) * a + j] = hi;
        }
    }
    __syncthreads();
    if (threadIdx.x < a) {
        const uint32_t j = threadIdx.x;
        tile_lo[(size_t)blockIdx.x * a + j] = fminf(fminf(wl[0][j], wl[1][j]), fminf(wl[2][j], wl[3][j]));
        tile_hi[(size_t)blockIdx.x * a + j] = fmaxf(fmaxf(wh[0][j], wh[1][j]), fmaxf(wh[2][j], wh[3][j]));
    }
}

__device__ __forceinline__ bool boxes_meet(const float* __restrict__ alo, const float* __restrict__ ahi,
                                           const float* __restrict__ blo, const float* __restrict__ bhi, uint32_t a) {
    bool ok = true;
    for (uint32_t j = 0; j < a; ++j) ok = ok && alo[j] <= bhi[j] && blo[j] <= ahi[j];
    return ok;
}

// Per query tile (256 threads): the point tiles whose attribute bounds meet the tile's union
// box, in increasing order.
__global__ void bf_tiles_kernel(const float* __restrict__ tbox, uint32_t a8, uint32_t tiles, uint32_t a,
                                const float* __restrict__ qlo, const float* __restrict__ qhi,
                                uint32_t* __restrict__ list, uint32_t* __restrict__ count,
                                unsigned int* __restrict__ products) {
    __shared__ uint32_t wc[8];
    const uint32_t qt = blockIdx.x, lane = lane_id(), w = threadIdx.x >> 5;
    const float* lo = qlo + (size_t)qt * a;
    const float* hi = qhi + (size_t)qt * a;
    uint32_t* out = list + (size_t)qt * tiles;
    uint32_t base = 0;
    for (uint32_t t0 = 0; t0 < tiles; t0 += blockDim.x) {
        const uint32_t t = t0 + threadIdx.x;
        const bool ok = t < tiles && boxes_meet(tbox + (size_t)t * 2 * a8, tbox + (size_t)t * 2 * a8 + a8, lo, hi, a);
        const uint32_t msk = __ballot_sync(kFull, ok);
        if (lane == 0) wc[w] = __popc(msk);
        __syncthreads();
        uint32_t before = 0, total = 0;
        for (uint32_t v = 0; v < (blockDim.x >> 5); ++v) {
            before += v < w ? wc[v] : 0u;
            total += wc[v];
        }
        if (ok) out[base + before + __popc(msk & lanemask_lt())] = t;
        base += total;
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        count[qt] = base;
        atomicAdd(products, base);
    }
}

// Per-thread candidate list: a max-heap of up to KM (a, position) entries in shared memory
// (entry i of owner o at i * OWN + o), so that an insertion costs at most log2(KM) steps
// whatever its rank -- the same for every lane of a warp.  heap_push: n < KM entries; the
// entry sifts up.  heap_replace: a full heap whose root (its largest a) is above aj; the root
// is replaced and sifts down.
template <uint32_t OWN>
__device__ __forceinline__ void heap_push(float aj, uint32_t pos, uint32_t n, uint32_t owner, float* la, uint32_t* lp) {
    uint32_t i = n;
#pragma unroll 1
    while (i > 0) {
        const uint32_t p = (i - 1) >> 1;
        const float ap = la[p * OWN + owner];
        if (!(ap < aj)) break;
        la[i * OWN + owner] = ap;
        lp[i * OWN + owner] = lp[p * OWN + owner];
        i = p;
    }
    la[i * OWN + owner] = aj;
    lp[i * OWN + owner] = pos;
}
template <uint32_t OWN>
__device__ __forceinline__ void heap_sift_down(float aj, uint32_t pos, uint32_t n, uint32_t owner, float* la,
                                               uint32_t* lp) {
    uint32_t i = 0;
#pragma unroll 1
    for (;;) {
        uint32_t c = 2 * i + 1;
        if (c >= n) break;
        float ac = la[c * OWN + owner];
        if (c + 1 < n) {
            const float a2 = la[(c + 1) * OWN + owner];
            if (a2 > ac) {
                ac = a2;
                ++c;
            }
        }
        if (!(ac > aj)) break;
        la[i * OWN + owner] = ac;
        lp[i * OWN + owner] = lp[c * OWN + owner];
        i = c;
    }
    la[i * OWN + owner] = aj;
    lp[i * OWN + owner] = pos;
}
// Heap of n entries -> ascending order in place (heapsort).
template <uint32_t OWN>
__device__ __noinline__ void heap_sort(uint32_t n, uint32_t owner, float* la, uint32_t* lp) {
    for (uint32_t end = n; end > 1; --end) {
        const float top = la[0 * OWN + owner];
        const uint32_t tp = lp[0 * OWN + owner];
        const float x = la[(end - 1) * OWN + owner];
        const uint32_t xp = lp[(end - 1) * OWN + owner];
        heap_sift_down<OWN>(x, xp, end - 1, owner, la, lp);
        la[(end - 1) * OWN + owner] = top;
        lp[(end - 1) * OWN + owner] = tp;
    }
}

struct TcArgs {
    const __half* at;        // query tiles
    const __half* xt;        // point tiles
    const float* px;         // per point position (padded)
    const float* pattrs;     // per row (padded with NaN), a per point
    const uint32_t* rowpos;  // per row: the point's position
    const float* tbox;       // point tiles x 2 x a8: attribute bounds (lo then hi) of each tile
    const float* glo;        // (query tiles * 4) x a: union box of each group of 32 rows
    const float* ghi;
    const float* lb;         // caller's boxes (original query order)
    const float* rb;
    const uint32_t* perm;    // sorted row -> query
    const uint32_t* flag;    // sorted row -> 0 = handled here
    const uint32_t* tl;      // query tiles x point tiles: relevant tiles
    const uint32_t* pre;     // query tiles + 1: exclusive prefix of the relevant-tile counts
    const uint32_t* sched;   // [0] total tile products W, [1] CTAs that take work G
    uint32_t* thr_g;         // per sorted row: smallest published list threshold (ordered bits)
    uint32_t* row_fb;        // per sorted row: 1 = answer on the CUDA cores
    uint2* cand;             // rows x LISTS x KM (a bits, position)
    uint32_t* cand_n;        // rows x LISTS (0 = empty, kEmpty = list not valid)
    uint32_t* timeouts;
    uint32_t qtiles, tiles, a, a8, dp, nck, stages, kc;  // kc: elements per stage (64 or 32)
    uint32_t stream_a;  // 1: the query tile's chunks are copied into every stage beside the point chunk
    uint32_t polls;     // bound of every barrier wait
    uint32_t extra_tx;  // test hook: bytes the query-tile load expects but never receives
};

// CTA c of G takes the tile products [W c / G, W (c + 1) / G) of the query-tile-major
// order; the CTA that holds product p:
__device__ __forceinline__ uint32_t range_start(uint32_t W, uint32_t G, uint32_t c) {
    return (uint32_t)((uint64_t)W * c / G);
}
__device__ __forceinline__ uint32_t cta_of(uint32_t W, uint32_t G, uint32_t p) {
    uint32_t c = (uint32_t)((uint64_t)p * G / W);
    while (c + 1 < G && range_start(W, G, c + 1) <= p) ++c;
    while (c > 0 && range_start(W, G, c) > p) --c;
    return c;
}

// Exclusive prefix of the per-query-tile counts and the number of CTAs that take work: at
// most `grid`, and few enough that no query tile spans more than kSlots CTAs.
__global__ void bf_sched_kernel(const uint32_t* __restrict__ cnt, uint32_t qtiles, uint32_t grid,
                                uint32_t* __restrict__ pre, uint32_t* __restrict__ sched) {
    if (threadIdx.x != 0) return;
    uint32_t acc = 0, mx = 0;
    for (uint32_t i = 0; i < qtiles; ++i) {
        pre[i] = acc;
        acc += cnt[i];
        mx = max(mx, cnt[i]);
    }
    pre[qtiles] = acc;
    uint32_t G = 0;
    if (acc) {
        const uint64_t cap = (uint64_t)(kSlots - 4) * acc / mx;
        G = (uint32_t)(cap < 1 ? 1 : (cap > grid ? grid : cap));
    }
    sched[0] = acc;
    sched[1] = G;
}

// Attribute bounds of a tile: lo[a8] then hi[a8] floats, a8 = a rounded up to 4 (16-byte rows).
__host__ __device__ inline uint32_t tbox_stride(uint32_t a) { return (a + 3) / 4 * 4; }

// Shared-memory layout of bf_tc_kernel (byte offsets from a 1024-aligned base).  A meta slot
// holds a tile's px (128 floats), its rows' positions (128), its points' attributes (128 x a
// floats) and the tile's attribute bounds (2 x a8 floats).
// With stream_a (rows wider than kResidentDp) there is no resident query tile: a stage holds
// the query tile's chunk (first half) and the point tile's chunk of the same K range.
struct TcLayout {
    uint32_t a_off, b_off, stage_bytes, meta_off, meta_bytes, la_off, lp_off, box_off, bar_off, total;
};
__host__ __device__ inline TcLayout tc_layout(uint32_t dp, uint32_t stages, uint32_t a, uint32_t stream_a, uint32_t km,
                                              uint32_t own, uint32_t kc) {
    TcLayout L;
    uint32_t o = 0;
    L.a_off = o;
    if (!stream_a) {
        o += kBM * dp * 2;
        o = (o + 1023u) & ~1023u;
    }
    L.b_off = o;
    L.stage_bytes = (stream_a ? 2u : 1u) * kBN * kc * 2;
    o += stages * L.stage_bytes;
    L.meta_off = o;
    L.meta_bytes = kBN * 4 * (2 + a) + 8 * tbox_stride(a);
    o += kMeta * L.meta_bytes;
    L.la_off = o;
    o += km * own * 4;
    L.lp_off = o;
    o += km * own * 4;
    L.box_off = o;
    o += 2 * a * own * 4;
    L.bar_off = o;
    o += (2 * stages + 2 * kAcc + 2 * kMeta + 3) * 8 + 16;
    L.total = o + 1024;  // room to align the base
    return L;
}

// The owner's box: NA attributes in registers (NA = 0: a attributes read from shared memory).
// Tests combine with & (no short-circuit branches).
template <int NA, uint32_t OWN>
struct OwnBox {
    float lo[NA > 0 ? NA : 1], hi[NA > 0 ? NA : 1];
    __device__ __forceinline__ void load(const float* blo, const float* bhi, uint32_t owner) {
#pragma unroll
        for (int e = 0; e < NA; ++e) {
            lo[e] = blo[e * OWN + owner];
            hi[e] = bhi[e * OWN + owner];
        }
    }
    __device__ __forceinline__ float l(uint32_t e, const float* blo, uint32_t owner) const {
        return NA > 0 ? lo[e] : blo[e * OWN + owner];
    }
    __device__ __forceinline__ float u(uint32_t e, const float* bhi, uint32_t owner) const {
        return NA > 0 ? hi[e] : bhi[e * OWN + owner];
    }
    // point attributes pa[0..a) inside the box
    __device__ __forceinline__ bool has(const float* pa, uint32_t a, const float* blo, const float* bhi,
                                        uint32_t owner) const {
        bool in = true;
        if (NA > 0) {
#pragma unroll
            for (int e = 0; e < NA; ++e) in = in & (pa[e] >= lo[e]) & (pa[e] <= hi[e]);
        } else {
            for (uint32_t e = 0; e < a; ++e)
                in = in & (pa[e] >= blo[e * OWN + owner]) & (pa[e] <= bhi[e * OWN + owner]);
        }
        return in;
    }
};

template <int NA, bool DEEP>
__global__ void __launch_bounds__(Lists<DEEP>::THREADS, 1) bf_tc_kernel(const __grid_constant__ TcArgs A) {
    using C = Lists<DEEP>;
    extern __shared__ unsigned char bf_smem_raw[];
    unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(bf_smem_raw) + 1023) & ~uintptr_t(1023));
    const TcLayout Lo = tc_layout(A.dp, A.stages, A.a, A.stream_a, C::KM, C::OWN, A.kc);
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + Lo.bar_off);
    uint64_t* full = bars;
    uint64_t* empty = full + A.stages;
    uint64_t* tfull = empty + A.stages;
    uint64_t* tempty = tfull + kAcc;
    uint64_t* mfull = tempty + kAcc;
    uint64_t* mempty = mfull + kMeta;
    uint64_t* aload = mempty + kMeta;
    uint64_t* afree = aload + 1;
    uint64_t* drain = afree + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile uint32_t* stop = tmem_slot + 1;
    float* la = reinterpret_cast<float*>(sm + Lo.la_off);
    uint32_t* lp = reinterpret_cast<uint32_t*>(sm + Lo.lp_off);
    float* blo = reinterpret_cast<float*>(sm + Lo.box_off);
    float* bhi = blo + A.a * C::OWN;
    const uint32_t a = NA > 0 ? (uint32_t)NA : A.a;

    const uint32_t warp = threadIdx.x >> 5, lane = lane_id();
    const uint32_t c = blockIdx.x, W = A.sched[0], G = A.sched[1];
    if (c >= G) return;  // uniform: this CTA takes no work (before any allocation)
    const uint32_t lo = range_start(W, G, c), hi = range_start(W, G, c + 1);
    if (lo >= hi) return;
    uint32_t qt0 = 0;  // query tile of product lo: the last with pre[qt] <= lo
    {
        uint32_t l = 0, h = A.qtiles;
        while (h - l > 1) {
            const uint32_t m = (l + h) >> 1;
            if (A.pre[m] <= lo)
                l = m;
            else
                h = m;
        }
        qt0 = l;
    }

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kAcc * kBN));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
    }
    if (threadIdx.x == 0) {
        for (uint32_t i = 0; i < A.stages; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        // a tile is read by the four epilogue warps of its parity (one per TMEM lane quarter)
        for (uint32_t i = 0; i < kAcc; ++i) {
            mbar_init(&tfull[i], 1);
            mbar_init(&tempty[i], 4);
        }
        for (uint32_t i = 0; i < kMeta; ++i) {
            mbar_init(&mfull[i], 1);
            mbar_init(&mempty[i], 4);
        }
        mbar_init(aload, 1);
        mbar_init(afree, 1);
        mbar_init(drain, 1);
        *stop = 0;
        fence_mbar_init();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t T = hi - lo;

    const uint32_t kc = A.kc;
    auto chunk_bytes = [&](uint32_t ch) { return kBN * min(kc, A.dp - ch * kc) * 2; };
    if (warp == 0) {
        // -------------------------------------------------------------- producer warp
        // Bulk copies: the query tile's rows (A), then per point tile its metadata slot and its
        // chunks into the stage ring.  Tile indices are read 32 at a time, one per lane.
        const size_t tile_halves = (size_t)kBN * A.dp;
        uint32_t pql = qt0, batch = 0xFFFFFFFFu, my_tile = 0;
        auto tile_of = [&](uint32_t t) {  // warp-collective
            if ((t & ~31u) != batch) {
                batch = t & ~31u;
                const uint32_t u = batch + lane;
                if (u < T) {
                    const uint32_t p = lo + u;
                    while (A.pre[pql + 1] <= p) ++pql;
                    my_tile = A.tl[(size_t)pql * A.tiles + (p - A.pre[pql])];
                }
            }
            return __shfl_sync(kFull, my_tile, t & 31u);
        };
        auto load_a = [&](uint32_t qt) {
            mbar_arrive_expect_tx(aload, kBM * A.dp * 2 + A.extra_tx);
            for (uint32_t ch = 0; ch < A.nck; ++ch)
                bulk_g2s(sm + Lo.a_off + ch * (kBM * kc * 2), A.at + (size_t)qt * kBM * A.dp + (size_t)ch * (kBM * kc),
                         chunk_bytes(ch), aload);
        };
        bool ok = true;
        uint32_t cq = qt0, na = 1, i = 0, nm = 0;  // A loads, chunks and metadata slots issued
        uint32_t pnext = A.pre[cq + 1];  // first product of the next query tile (read once per tile change)
        if (lane == 0 && !A.stream_a) load_a(qt0);
        for (uint32_t t = 0; ok && t < T; ++t) {
            const uint32_t tile = tile_of(t);
            const uint32_t qprev = cq;
            while (pnext <= lo + t) pnext = A.pre[++cq + 1];
            if (cq != qprev && !A.stream_a) {
                // a new query tile: its rows replace A once the MMAs of the previous one are done
                ok = __all_sync(kFull, bwait(afree, (na - 1) & 1u, stop, A.polls));
                if (!ok) break;
                if (lane == 0) load_a(cq);
                ++na;
            }
            const uint32_t m = t % kMeta;
            if (t >= kMeta && !(ok = __all_sync(kFull, bwait(&mempty[m], ((t / kMeta) - 1) & 1u, stop, A.polls)))) break;
            if (lane == 0) {
                fence_proxy_async_smem();  // the epilogue's reads of this slot come before the copy
                unsigned char* slot = sm + Lo.meta_off + m * Lo.meta_bytes;
                mbar_arrive_expect_tx(&mfull[m], Lo.meta_bytes);
                bulk_g2s(slot, A.px + (size_t)tile * kBN, kBN * 4, &mfull[m]);
                bulk_g2s(slot + kBN * 4, A.rowpos + (size_t)tile * kBN, kBN * 4, &mfull[m]);
                bulk_g2s(slot + kBN * 8, A.pattrs + (size_t)tile * kBN * a, kBN * 4 * a, &mfull[m]);
                bulk_g2s(slot + kBN * 4 * (2 + a), A.tbox + (size_t)tile * 2 * A.a8, 8 * A.a8, &mfull[m]);
            }
            ++nm;
            for (uint32_t ch = 0; ch < A.nck; ++ch, ++i) {
                const uint32_t st = i % A.stages;
                if (i >= A.stages && !(ok = __all_sync(kFull, bwait(&empty[st], ((i / A.stages) - 1) & 1u, stop, A.polls))))
                    break;
                if (lane == 0) {
                    const uint32_t bytes = chunk_bytes(ch);
                    unsigned char* stg = sm + Lo.b_off + st * Lo.stage_bytes;
                    if (A.stream_a) {
                        mbar_arrive_expect_tx(&full[st], 2 * bytes + A.extra_tx);
                        bulk_g2s(stg, A.at + (size_t)cq * kBM * A.dp + (size_t)ch * (kBM * kc), bytes, &full[st]);
                        stg += kBN * kc * 2;
                    } else {
                        mbar_arrive_expect_tx(&full[st], bytes);
                    }
                    bulk_g2s(stg, A.xt + tile * tile_halves + (size_t)ch * (kBN * kc), bytes, &full[st]);
                }
            }
        }
        if (!ok) *stop = 1u;
        // every copy issued lands before the CTA exits: the last load of each stage, each
        // metadata slot and A (bounded waits; in normal operation these completed long ago)
        if (lane == 0) {
            for (uint32_t st = 0; st < A.stages && st < i; ++st) {
                const uint32_t last = st + ((i - 1 - st) / A.stages) * A.stages;
                uint32_t p = 0;
                while (!mbar_try_wait(&full[st], (last / A.stages) & 1u, 1000) && ++p < A.polls) {
                }
            }
            for (uint32_t m = 0; m < kMeta && m < nm; ++m) {
                const uint32_t last = m + ((nm - 1 - m) / kMeta) * kMeta;
                uint32_t p = 0;
                while (!mbar_try_wait(&mfull[m], (last / kMeta) & 1u, 1000) && ++p < A.polls) {
                }
            }
            uint32_t p = 0;
            while (!A.stream_a && !mbar_try_wait(aload, (na - 1) & 1u, 1000) && ++p < A.polls) {
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // -------------------------------------------------------------- MMA warp
        if (lane == 0) {
            const unsigned char* sA = sm + Lo.a_off;
            const unsigned char* sB = sm + Lo.b_off;
            bool ok = true;
            uint32_t cq = qt0, na = 0, i = 0;
            uint32_t pnext = A.pre[cq + 1];  // first product of the next query tile
            for (uint32_t t = 0; t < T; ++t) {
                const uint32_t b = t % kAcc;
                const uint32_t qprev = cq;
                while (pnext <= lo + t) pnext = A.pre[++cq + 1];
                if (!A.stream_a && (t == 0 || cq != qprev)) {
                    if (!(ok = bwait(aload, na & 1u, stop, A.polls))) break;
                    ++na;
                }
                if (t >= kAcc && !(ok = bwait(&tempty[b], ((t / kAcc) - 1) & 1u, stop, A.polls))) break;
                tc_fence_after();
                for (uint32_t ch = 0; ch < A.nck; ++ch, ++i) {
                    const uint32_t st = i % A.stages;
                    if (!(ok = bwait(&full[st], (i / A.stages) & 1u, stop, A.polls))) break;
                    tc_fence_after();
                    const uint32_t ksteps = min(kc, A.dp - ch * kc) / 16;
                    const uint32_t sst = smem_u32(sB + st * Lo.stage_bytes);
                    const uint32_t a0 = A.stream_a ? sst : smem_u32(sA + ch * (kBM * kc * 2));
                    const uint32_t b0 = A.stream_a ? sst + kBN * kc * 2 : sst;
                    for (uint32_t s = 0; s < ksteps; ++s)
                        mma_f16(tmem + b * kBN, kmajor_desc(a0 + s * 2 * kColBytes, kColBytes, 128),
                                kmajor_desc(b0 + s * 2 * kColBytes, kColBytes, 128), (ch | s) ? 1u : 0u);
                    mma_commit(&empty[st]);  // the stage is free once these MMAs have read it
                }
                if (!ok) break;
                mma_commit(&tfull[b]);
                if (!A.stream_a && (t + 1 == T || pnext <= lo + t + 1))
                    mma_commit(afree);  // last tile of this query tile
            }
            if (!ok) *stop = 1u;
            // every MMA has completed before TMEM is released
            mma_commit(drain);
            uint32_t p = 0;
            while (!mbar_try_wait(drain, 0, 1000) && ++p < A.polls) {
            }
            if (p >= A.polls) *stop = 1u;
        }
        __syncwarp();
    } else {
        // -------------------------------------------------------------- epilogue warps
        // warp: TMEM lane quarter qq (rows 32 qq ..), tiles of parity h
        const uint32_t ew = warp - 2, qq = warp & 3u, h = ew >> 2;
        const uint32_t row = qq * 32 + lane, owner = ew * 32 + lane;
        bool ok = true;
        uint32_t t = 0, cq = qt0;
        // one segment per query tile met in [lo, hi)
        while (t < T) {
            while (A.pre[cq + 1] <= lo + t) ++cq;
            const uint32_t seg_end = min(hi, A.pre[cq + 1]) - lo;
            const uint32_t r = cq * kBM + row;
            const uint32_t slot_id = c - cta_of(W, G, A.pre[cq]);
            const uint32_t q = A.perm[r];
            bool valid = A.flag[r] == 0;  // a query handled here with a box that is not empty
            for (uint32_t j = 0; valid && j < a; ++j) valid = A.lb[(size_t)q * a + j] <= A.rb[(size_t)q * a + j];
            for (uint32_t j = 0; j < a; ++j) {
                blo[j * C::OWN + owner] = valid ? A.lb[(size_t)q * a + j] : __int_as_float(0x7f800000);
                bhi[j * C::OWN + owner] = valid ? A.rb[(size_t)q * a + j] : -__int_as_float(0x7f800000);
            }
            OwnBox<NA, C::OWN> box;
            box.load(blo, bhi, owner);
            float glo[kMaxAttr], ghi[kMaxAttr];  // union box of this warp's 32 rows (warp-uniform)
#pragma unroll
            for (uint32_t j = 0; j < kMaxAttr; ++j) {
                glo[j] = j < a ? A.glo[((size_t)cq * 4 + qq) * a + j] : -__int_as_float(0x7f800000);
                ghi[j] = j < a ? A.ghi[((size_t)cq * 4 + qq) * a + j] : __int_as_float(0x7f800000);
            }
            uint32_t n = 0;
            float thr = __int_as_float(0x7f800000);
            uint32_t pub = __ldcg(A.thr_g + r);
            for (; t < seg_end; ++t) {
                if (C::NPAR == 2 && (t & 1u) != h) continue;  // the other warp of this lane quarter takes it
                const uint32_t b = t % kAcc, m = t % kMeta;
                ok = bwait(&mfull[m], (t / kMeta) & 1u, stop, A.polls) && bwait(&tfull[b], (t / kAcc) & 1u, stop, A.polls);
                if (!__all_sync(kFull, ok)) {
                    ok = false;
                    break;
                }
                // a tighter threshold published by another list of this query (any full list's
                // largest entry bounds the query's KM smallest); the next one is fetched now
                thr = fminf(thr, ord2f(pub));
                pub = __ldcg(A.thr_g + r);
                tc_fence_after();
                const unsigned char* slot = sm + Lo.meta_off + m * Lo.meta_bytes;
                const float* mpx = reinterpret_cast<const float*>(slot);
                const uint32_t* mpos = reinterpret_cast<const uint32_t*>(slot) + kBN;
                const float* mat = mpx + 2 * kBN;
                const float* tlo = mpx + kBN * (2 + a);
                const float* thi = tlo + A.a8;
                bool wrel = true;
#pragma unroll
                for (uint32_t j = 0; j < kMaxAttr; ++j)
                    if (j < a) wrel = wrel & (tlo[j] <= ghi[j]) & (glo[j] <= thi[j]);
                if (wrel) {
                    // mine: the tile meets the row's box; inside: it lies within it (no point
                    // needs a test)
                    bool mine = valid, inside = valid;
                    for (uint32_t j = 0; j < a; ++j) {
                        const float bl = box.l(j, blo, owner), bu = box.u(j, bhi, owner);
                        mine = mine & (tlo[j] <= bu) & (bl <= thi[j]);
                        inside = inside & (bl <= tlo[j]) & (thi[j] <= bu);
                    }
                    const uint32_t taddr = tmem + ((qq * 32u) << 16) + b * kBN;
                    uint32_t v[2][32];
                    __syncwarp();  // tcgen05.ld is warp-collective
                    tmem_ld32(taddr, v[0]);
                    tmem_wait_ld(v[0]);
#pragma unroll
                    for (uint32_t g = 0; g < 4; ++g) {
                        const uint32_t col = g * 32, cur = g & 1u;
                        // the next 32 columns load while these are processed
                        if (g + 1 < 4) tmem_ld32(taddr + col + 32, v[cur ^ 1u]);
                        uint32_t mask = 0;
                        float av[32];
                        if (mine) {
                            const float4* pm = reinterpret_cast<const float4*>(mpx + col);
#pragma unroll
                            for (uint32_t j4 = 0; j4 < 8; ++j4) {
                                const float4 p4 = pm[j4];
                                av[4 * j4 + 0] = fmaf(-2.0f, __uint_as_float(v[cur][4 * j4 + 0]), p4.x);
                                av[4 * j4 + 1] = fmaf(-2.0f, __uint_as_float(v[cur][4 * j4 + 1]), p4.y);
                                av[4 * j4 + 2] = fmaf(-2.0f, __uint_as_float(v[cur][4 * j4 + 2]), p4.z);
                                av[4 * j4 + 3] = fmaf(-2.0f, __uint_as_float(v[cur][4 * j4 + 3]), p4.w);
                            }
                            // points below the threshold (four independent partial masks)
                            uint32_t m4[4] = {0u, 0u, 0u, 0u};
#pragma unroll
                            for (uint32_t j = 0; j < 32; ++j) m4[j & 3] |= (uint32_t)(av[j] < thr) << j;
                            mask = (m4[0] | m4[1]) | (m4[2] | m4[3]);
                        }
                        // rows whose box does not contain the tile test only those points
                        uint32_t todo = inside ? 0u : mask;
                        if (!inside) mask = 0;
                        while (__any_sync(kFull, todo != 0)) {
                            if (todo) {
                                const uint32_t j = __ffs(todo) - 1;
                                todo &= todo - 1;
                                if (box.has(mat + (col + j) * a, a, blo, bhi, owner)) mask |= 1u << j;
                            }
                        }
                        // insertion rounds: every lane with candidates left takes its lowest one
                        const float before = thr;
                        while (__any_sync(kFull, mask != 0)) {
                            if (mask) {
                                const uint32_t j = __ffs(mask) - 1;
                                mask &= mask - 1;
                                // av[j] for the lane's own j: a five-level select tree (31
                                // selects, five deep, instead of a chain 31 deep)
                                float s16[16], s8[8], s4[4], s2[2];
#pragma unroll
                                for (uint32_t u = 0; u < 16; ++u) s16[u] = (j & 16u) ? av[u + 16] : av[u];
#pragma unroll
                                for (uint32_t u = 0; u < 8; ++u) s8[u] = (j & 8u) ? s16[u + 8] : s16[u];
#pragma unroll
                                for (uint32_t u = 0; u < 4; ++u) s4[u] = (j & 4u) ? s8[u + 4] : s8[u];
#pragma unroll
                                for (uint32_t u = 0; u < 2; ++u) s2[u] = (j & 2u) ? s4[u + 2] : s4[u];
                                const float aj = (j & 1u) ? s2[1] : s2[0];
                                if (aj < thr) {
                                    const uint32_t pos = mpos[col + j];
                                    if (n < C::KM) {
                                        heap_push<C::OWN>(aj, pos, n, owner, la, lp);
                                        if (++n == C::KM) thr = fminf(thr, la[owner]);
                                    } else {
                                        heap_sift_down<C::OWN>(aj, pos, C::KM, owner, la, lp);
                                        thr = fminf(thr, la[owner]);
                                    }
                                }
                            }
                        }
                        if (thr < before) atomicMin(A.thr_g + r, f2ord(thr));
                        if (g + 1 < 4) {
                            __syncwarp();
                            tmem_wait_ld(v[cur ^ 1u]);
                        }
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&tempty[b]);
                    mbar_arrive(&mempty[m]);
                }
            }
            // this segment's list of row r (slot slot_id, tile parity h)
            heap_sort<C::OWN>(n, owner, la, lp);
            if (slot_id < kSlots) {
                const uint32_t l = slot_id * C::NPAR + h;
                uint2* out = A.cand + ((size_t)r * C::LISTS + l) * C::KM;
                for (uint32_t k = 0; k < n; ++k)
                    out[k] = make_uint2(__float_as_uint(la[k * C::OWN + owner]), lp[k * C::OWN + owner]);
                A.cand_n[(size_t)r * C::LISTS + l] = (ok && !*stop) ? n : kEmpty;
            } else {
                A.row_fb[r] = 1u;  // more CTAs than list slots met this query tile
            }
            if (!ok) break;
        }
        if (!ok || *stop) {
            // rows of the segments this warp did not finish go to the CUDA cores
            for (uint32_t u = t; u < T;) {
                while (A.pre[cq + 1] <= lo + u) ++cq;
                A.row_fb[cq * kBM + row] = 1u;
                u = min(hi, A.pre[cq + 1]) - lo;
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    __syncwarp();
    if (threadIdx.x == 0 && *stop) atomicAdd(A.timeouts, 1u);
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kAcc * kBN));
}

struct MergeArgs {
    const uint2* cand;
    const uint32_t* cand_n;
    const uint32_t* perm;
    const uint32_t* flag;
    const uint32_t* row_fb;
    const float* pq;
    const float* dq;
    const float* queries;
    const float4* vec32;
    const uint32_t* i2g;
    uint32_t* ids;
    float* dists;
    uint32_t* fb_list;
    uint32_t* fb_cnt;
    uint32_t qpad, dim, nch, k, test_every;
    float inv_s, dmax;
    double eta;
};

// One warp per sorted row: merge, exact re-rank, proof (see the file comment).  The KM
// smallest a of the merged lists are re-ranked (KM / 32 per lane); the k smallest canonical
// keys are the answer when the bound proves that no point left out can beat the k-th.
template <bool DEEP>
__global__ void __launch_bounds__(256) bf_merge_kernel(const __grid_constant__ MergeArgs M) {
    using C = Lists<DEEP>;
    constexpr uint32_t NR = C::KM / 32;  // re-ranked candidates per lane
    extern __shared__ __align__(16) float mq[];
    const uint32_t lane = lane_id(), w = threadIdx.x >> 5;
    const uint32_t r = blockIdx.x * (blockDim.x >> 5) + w;
    if (r >= M.qpad) return;
    const uint32_t q = M.perm[r];
    if (q == kEmpty) return;
    bool fallback = M.flag[r] != 0 || M.row_fb[r] != 0 || (M.test_every && q % M.test_every == 0);
    const uint32_t nl = C::LISTS;
    const uint32_t cnt = lane < nl ? M.cand_n[(size_t)r * nl + lane] : 0u;
    fallback = fallback || __any_sync(kFull, cnt == kEmpty);
    if (!fallback) {
        float4* qs = reinterpret_cast<float4*>(mq + (size_t)w * M.nch * 4);
        float* qf = reinterpret_cast<float*>(qs);
        for (uint32_t i = lane; i < M.nch * 4; i += 32) qf[i] = i < M.dim ? M.queries[(size_t)q * M.dim + i] : 0.0f;
        const uint2* lst = M.cand + ((size_t)r * nl + (lane < nl ? lane : 0u)) * C::KM;
        uint32_t hd = 0;
        const uint32_t inf_o = f2ord(__int_as_float(0x7f800000));
        uint32_t head = (lane < nl && cnt > 0) ? f2ord(__uint_as_float(lst[0].x)) : inf_o;
        const uint32_t lthr = (lane < nl && cnt == C::KM) ? f2ord(__uint_as_float(lst[C::KM - 1].x)) : inf_o;
        uint32_t astar = __reduce_min_sync(kFull, lthr);
        uint32_t mypos[NR];
#pragma unroll
        for (uint32_t i = 0; i < NR; ++i) mypos[i] = kEmpty;
        uint32_t npick = 0;
        for (; npick < C::KM; ++npick) {
            const uint32_t mn = __reduce_min_sync(kFull, head);
            if (mn == inf_o) break;
            const uint32_t win = __ffs(__ballot_sync(kFull, head == mn)) - 1;
            const uint32_t p = __shfl_sync(kFull, lane == win ? lst[hd].y : 0u, win);
            if (lane == (npick & 31u)) {
#pragma unroll
                for (uint32_t i = 0; i < NR; ++i)
                    if (i == (npick >> 5)) mypos[i] = p;
            }
            if (lane == win) {
                ++hd;
                head = hd < cnt ? f2ord(__uint_as_float(lst[hd].x)) : inf_o;
            }
        }
        if (npick == C::KM) astar = min(astar, __reduce_min_sync(kFull, head));
        __syncwarp();
        key_t key[NR];
#pragma unroll
        for (uint32_t i = 0; i < NR; ++i) {
            key[i] = kEmptyKey;
            if (i * 32 + lane < npick) {
                const float c = dist32(M.vec32 + (size_t)mypos[i] * M.nch, qs, M.nch);
                key[i] = ((key_t)__float_as_uint(c) << 32) | __ldg(M.i2g + mypos[i]);
            }
        }
        // res[i] of lane l: the (32 i + l)-th smallest key; kth: the k-th smallest
        key_t res[NR], kth;
        if (NR == 1) {
            res[0] = warp_sort32_key(key[0]);
            kth = __shfl_sync(kFull, res[0], M.k - 1);
        } else {
            // the lane's keys ascending, then k rounds that take the warp's smallest head
#pragma unroll
            for (uint32_t i = 0; i < NR; ++i)
#pragma unroll
                for (uint32_t j = 0; j + 1 < NR - i; ++j)
                    if (key[j] > key[j + 1]) {
                        const key_t t = key[j];
                        key[j] = key[j + 1];
                        key[j + 1] = t;
                    }
#pragma unroll
            for (uint32_t i = 0; i < NR; ++i) res[i] = kEmptyKey;
            kth = kEmptyKey;
            for (uint32_t i = 0; i < M.k; ++i) {
                const uint32_t hi = __reduce_min_sync(kFull, (uint32_t)(key[0] >> 32));
                const uint32_t lo = __reduce_min_sync(kFull, (uint32_t)(key[0] >> 32) == hi ? (uint32_t)key[0] : ~0u);
                const key_t mn = ((key_t)hi << 32) | lo;
                kth = mn;
                if (mn == kEmptyKey) break;
                if (lane == (i & 31u)) {
#pragma unroll
                    for (uint32_t j = 0; j < NR; ++j)
                        if (j == (i >> 5)) res[j] = mn;
                }
                const uint32_t win = __ffs(__ballot_sync(kFull, key[0] == mn)) - 1;
                if (lane == win) {
#pragma unroll
                    for (uint32_t j = 0; j + 1 < NR; ++j) key[j] = key[j + 1];
                    key[NR - 1] = kEmptyKey;
                }
            }
        }
        if (astar != inf_o) {
            // some point was left out: it must provably lose to the k-th re-ranked one
            bool proven = false;
            if (kth != kEmptyKey) {
                const double as = (double)ord2f(astar);
                const double tlo = (double)M.pq[r] + as - fabs(as) * 0x1p-22;
                double t = (tlo > 0.0 ? sqrt(tlo) * (double)M.inv_s : 0.0) - (double)M.dq[r] - (double)M.dmax;
                t = t > 0.0 ? t * (1.0 - 1e-12) : 0.0;
                const double lbd = t * t * (1.0 - M.eta);
                proven = lbd > (double)key_dist(kth);
            }
            fallback = !proven;
        }
        if (!fallback) {
#pragma unroll
            for (uint32_t i = 0; i < NR; ++i) {
                const uint32_t j = i * 32 + lane;
                if (j < M.k) {
                    M.ids[(size_t)q * M.k + j] = res[i] == kEmptyKey ? kEmpty : (uint32_t)res[i];
                    if (M.dists)
                        M.dists[(size_t)q * M.k + j] = res[i] == kEmptyKey ? __int_as_float(0x7f800000) : key_dist(res[i]);
                }
            }
        }
    }
    if (fallback && lane == 0) M.fb_list[atomicAdd(M.fb_cnt, 1u)] = q;
}

// Workspace of one call, carved out of one stream-ordered allocation.
struct Carve {
    unsigned char* base = nullptr;
    size_t used = 0;
    template <typename T>
    T* take(size_t count) {
        const size_t off = (used + 255) & ~size_t(255);
        used = off + std::max<size_t>(count, 1) * sizeof(T);
        return base ? reinterpret_cast<T*>(base + off) : nullptr;
    }
};

double kappa_of(uint32_t dp) { return (2.0 * dp + 64.0) * 0x1p-23; }

// Origin and inverse extent of each attribute: the outer bounds of the grid's slices.
std::vector<float> attr_range(const DeviceIndex& d) {
    std::vector<float> ar(2 * d.a);
    uint32_t off = 0;
    for (uint32_t j = 0; j < d.a; ++j) {
        const float lo = d.lq[off], hi = d.rq[off + d.grid[j] - 1];
        ar[j] = lo;
        ar[d.a + j] = hi > lo ? 1.0f / (hi - lo) : 0.0f;
        off += d.grid[j];
    }
    return ar;
}

}  // namespace

void free_bf_tc(DeviceIndex& d) {
    if (d.bf_ws_ev) {
        cudaEventSynchronize(d.bf_ws_ev);
        cudaEventDestroy(d.bf_ws_ev);
        d.bf_ws_ev = nullptr;
    }
    if (d.bf_ws) cudaFree(d.bf_ws);
    d.bf_ws = nullptr;
    d.bf_ws_bytes = 0;
    void* ptrs[] = {d.bf_x, d.bf_px, d.bf_mean, d.bf_tbox, d.bf_attrs, d.bf_rowpos, d.bf_arange, d.bf_tcnt,
                    d.bf_sbox, d.bf_scnt};
    for (void* p : ptrs)
        if (p) cudaFree(p);
    d.bf_x = nullptr;
    d.bf_px = d.bf_mean = d.bf_tbox = d.bf_attrs = d.bf_arange = d.bf_sbox = nullptr;
    d.bf_rowpos = d.bf_tcnt = d.bf_scnt = nullptr;
    d.bf_ok = false;
    d.at_ok = false;
}

namespace {
__global__ void super_tile_kernel(const float* __restrict__ tbox, const uint32_t* __restrict__ tcnt, uint32_t tiles,
                                  uint32_t a8, uint32_t stiles, float* __restrict__ sbox, uint32_t* __restrict__ scnt);
}  // namespace

// Attribute tiles (every index): rows in the Morton order of their attributes, 128 per
// tile, each tile's attribute bounds and the tile-padded attribute copy.  Used by the
// tensor-core brute force and by the plan's box counts.
gf_status attr_tiles_prepare(DeviceIndex& d) {
    d.at_ok = false;
    if (d.n == 0 || d.a == 0 || d.a > kMaxAttr) return GF_OK;
    const uint32_t tiles = (d.n + kBN - 1) / kBN, npad = tiles * kBN;
    gf_status st = GF_OK;
    auto ck = [&](cudaError_t e, const char* what) {
        if (e != cudaSuccess && st == GF_OK) st = cuda_fail(e, what);
        return st == GF_OK;
    };
    do {
        if (!ck(cudaMalloc((void**)&d.bf_tbox, sizeof(float) * (size_t)tiles * 2 * tbox_stride(d.a)), "tile bounds"))
            break;
        if (!ck(cudaMalloc((void**)&d.bf_attrs, sizeof(float) * (size_t)npad * d.a), "tile attributes")) break;
        if (!ck(cudaMalloc((void**)&d.bf_rowpos, sizeof(uint32_t) * (size_t)npad), "tile positions")) break;
        if (!ck(cudaMalloc((void**)&d.bf_arange, sizeof(float) * 2 * d.a), "attribute range")) break;
        if (!ck(cudaMalloc((void**)&d.bf_tcnt, sizeof(uint32_t) * tiles), "tile counts")) break;
        const uint32_t stiles = (tiles + kSuperTiles - 1) / kSuperTiles;  // super-tiles (box counts)
        if (!ck(cudaMalloc((void**)&d.bf_sbox, sizeof(float) * (size_t)stiles * 2 * tbox_stride(d.a)), "super-tiles"))
            break;
        if (!ck(cudaMalloc((void**)&d.bf_scnt, sizeof(uint32_t) * stiles), "super-tiles")) break;
        {
            std::vector<float> ar = attr_range(d);
            if (!ck(cudaMemcpy(d.bf_arange, ar.data(), sizeof(float) * 2 * d.a, cudaMemcpyHostToDevice), "range"))
                break;
        }
        // row order: Morton order of the points' attributes
        unsigned long long *k0 = nullptr, *k1 = nullptr;
        uint32_t* v0 = nullptr;
        void* tmp = nullptr;
        size_t tb = 0;
        cub::DeviceRadixSort::SortPairs(nullptr, tb, k0, k1, v0, v0, (int)d.n);
        bool good = ck(cudaMalloc((void**)&k0, 8 * (size_t)d.n), "tile sort") &&
                    ck(cudaMalloc((void**)&k1, 8 * (size_t)d.n), "tile sort") &&
                    ck(cudaMalloc((void**)&v0, 4 * (size_t)d.n), "tile sort") &&
                    ck(cudaMalloc(&tmp, std::max<size_t>(tb, 16)), "tile sort");
        if (good) {
            bf_point_keys_kernel<<<(d.n + 255) / 256, 256>>>(d.attrs, d.n, d.a, d.bf_arange, d.bf_arange + d.a, k0, v0);
            ck(cub::DeviceRadixSort::SortPairs(tmp, tb, k0, k1, v0, d.bf_rowpos, (int)d.n), "tile sort");
            // rowpos: sorted positions, then padding marks past n
            bf_tilebox_kernel<<<(tiles + 7) / 8, 256>>>(d.attrs, d.n, d.a, tbox_stride(d.a), tiles, d.bf_rowpos,
                                                        d.bf_tbox, d.bf_attrs, d.bf_rowpos, d.bf_tcnt);
            super_tile_kernel<<<(stiles + 7) / 8, 256>>>(d.bf_tbox, d.bf_tcnt, tiles, tbox_stride(d.a), stiles,
                                                         d.bf_sbox, d.bf_scnt);
            ck(cudaGetLastError(), "tile bounds");
            ck(cudaDeviceSynchronize(), "tile sort");
        }
        for (void* pp : {(void*)k0, (void*)k1, (void*)v0, tmp})
            if (pp) cudaFree(pp);
        if (st != GF_OK) break;
        d.bf_tiles = tiles;
        d.bf_stiles = stiles;
        d.bytes += sizeof(float) * (size_t)stiles * 2 * tbox_stride(d.a) + sizeof(uint32_t) * stiles + sizeof(float) * (size_t)tiles * 2 * tbox_stride(d.a) + sizeof(float) * (size_t)npad * d.a +
                   sizeof(uint32_t) * (size_t)npad + sizeof(float) * 2 * d.a + sizeof(uint32_t) * tiles;
        d.at_ok = true;
    } while (0);
    if (st != GF_OK) free_bf_tc(d);
    return st;
}

gf_status bf_tc_prepare(DeviceIndex& d) {
    d.bf_ok = false;
    if (!d.vec32 || d.n == 0 || !d.at_ok) return GF_OK;
    const uint32_t dp = (d.dim + 15) / 16 * 16;
    if (dp > kMaxDp) return GF_OK;  // wider rows use the CUDA-core kernel
    const uint32_t tiles = d.bf_tiles, npad = tiles * kBN;
    const float* x = reinterpret_cast<const float*>(d.vec32);
    double* sum = nullptr;
    uint32_t* words = nullptr;
    gf_status st = GF_OK;
    auto ck = [&](cudaError_t e, const char* what) {
        if (e != cudaSuccess && st == GF_OK) st = cuda_fail(e, what);
        return st == GF_OK;
    };
    do {
        if (!ck(cudaMalloc((void**)&sum, sizeof(double) * d.dim), "bf mean")) break;
        if (!ck(cudaMalloc((void**)&words, 16), "bf words")) break;
        if (!ck(cudaMalloc((void**)&d.bf_mean, sizeof(float) * d.dim), "bf mean")) break;
        if (!ck(cudaMalloc((void**)&d.bf_x, sizeof(__half) * (size_t)npad * dp), "bf tiles")) break;
        if (!ck(cudaMalloc((void**)&d.bf_px, sizeof(float) * npad), "bf px")) break;
        ck(cudaMemset(sum, 0, sizeof(double) * d.dim), "bf mean");
        ck(cudaMemset(words, 0, 16), "bf words");
        const uint32_t blocks = std::min<uint32_t>(1024, (d.n + 255) / 256);
        bf_colsum_kernel<<<blocks, 128>>>(x, d.n, d.d4, d.dim, sum);
        std::vector<double> sh(d.dim);
        if (!ck(cudaMemcpy(sh.data(), sum, sizeof(double) * d.dim, cudaMemcpyDeviceToHost), "bf mean")) break;
        std::vector<float> mh(d.dim);
        for (uint32_t i = 0; i < d.dim; ++i) mh[i] = (float)(sh[i] / d.n);
        if (!ck(cudaMemcpy(d.bf_mean, mh.data(), sizeof(float) * d.dim, cudaMemcpyHostToDevice), "bf mean")) break;
        bf_maxabs_kernel<<<148 * 8, 256>>>(x, d.n, d.d4, d.dim, d.bf_mean, words, words + 1);
        uint32_t wh[2];
        if (!ck(cudaMemcpy(wh, words, 8, cudaMemcpyDeviceToHost), "bf range")) break;
        if (wh[1]) break;  // non-finite rows: the CUDA-core kernel ranks them
        float maxabs;
        std::memcpy(&maxabs, &wh[0], 4);
        int e = 0;
        std::frexp(maxabs > 0.0f ? maxabs : 1.0f, &e);  // maxabs < 2^e
        const int ex = std::min(100, std::max(-100, 14 - e));
        const float s = std::ldexp(1.0f, ex);
        // rows in the attribute tiles' order (rowpos: the sorted positions; padding rows past n)
        bf_convert_kernel<<<148 * 16, 256>>>(x, d.n, d.d4, d.dim, dp, d.bf_mean, s, 1.0 - kappa_of(dp), npad,
                                             d.bf_rowpos, reinterpret_cast<__half*>(d.bf_x), d.bf_px, words + 2);
        if (!ck(cudaMemcpy(wh, words + 2, 4, cudaMemcpyDeviceToHost), "bf residuals")) break;
        if (!ck(cudaGetLastError(), "bf prepare")) break;
        std::memcpy(&d.bf_dmax, &wh[0], 4);
        d.bf_scale = s;
        d.bf_dp = dp;
        d.bytes += sizeof(float) * d.dim + sizeof(__half) * (size_t)npad * dp + sizeof(float) * npad;
        d.bf_ok = std::isfinite(d.bf_dmax);
    } while (0);
    if (sum) cudaFree(sum);
    if (words) cudaFree(words);
    if (st != GF_OK || !d.bf_ok) {  // the attribute tiles stay; only the fp16 copy goes
        void* ptrs[] = {d.bf_x, d.bf_px, d.bf_mean};
        for (void* p : ptrs)
            if (p) cudaFree(p);
        d.bf_x = nullptr;
        d.bf_px = d.bf_mean = nullptr;
        d.bf_ok = false;
    }
    return st;
}

namespace {
constexpr uint32_t kSuper = kSuperTiles;  // tiles per super-tile of the box counts

// Bounds and counts of each super-tile (kSuper consecutive tiles, one warp each).
__global__ void super_tile_kernel(const float* __restrict__ tbox, const uint32_t* __restrict__ tcnt, uint32_t tiles,
                                  uint32_t a8, uint32_t stiles, float* __restrict__ sbox, uint32_t* __restrict__ scnt) {
    const uint32_t lane = lane_id();
    const uint32_t st = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (st >= stiles) return;
    const uint32_t t = st * kSuper + lane;
    uint32_t c = t < tiles ? tcnt[t] : 0u;
    for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(kFull, c, o);
    if (lane == 0) scnt[st] = c;
    for (uint32_t j = 0; j < a8; ++j) {
        float lo = t < tiles ? tbox[(size_t)t * 2 * a8 + j] : __int_as_float(0x7f800000);
        float hi = t < tiles ? tbox[(size_t)t * 2 * a8 + a8 + j] : -__int_as_float(0x7f800000);
        for (int o = 16; o > 0; o >>= 1) {
            lo = fminf(lo, __shfl_xor_sync(kFull, lo, o));
            hi = fmaxf(hi, __shfl_xor_sync(kFull, hi, o));
        }
        if (lane == 0) {
            sbox[(size_t)st * 2 * a8 + j] = lo;
            sbox[(size_t)st * 2 * a8 + a8 + j] = hi;
        }
    }
}

// Whether bounds [b, b + a8) .. [b + a8, b + 2 a8) meet / lie inside the box (a attributes).
__device__ __forceinline__ void meet_inside(const float* b, uint32_t a, uint32_t a8, const float* lo, const float* hi,
                                            bool& meet, bool& inside) {
    meet = inside = true;
#pragma unroll
    for (uint32_t j = 0; j < kMaxAttr; ++j) {
        if (j < a) {
            const float tl = b[j], th = b[a8 + j];
            meet = meet & (tl <= hi[j]) & (lo[j] <= th);
            inside = inside & (lo[j] <= tl) & (th <= hi[j]);
        }
    }
    inside = inside & meet;
}

// Points inside each query box (prefiltering_tag_elements, real_dataset_adapter.cuh:347-387)
// from the attribute tiles, one warp per query, two levels: super-tiles (32 consecutive
// tiles of the attribute-Morton order) then tiles.  A (super-)tile that lies inside the box
// adds its count of points with numeric attributes; one that meets the box without lying
// inside it is opened (its tiles, or its 128 rows, 4 per lane); the others add nothing.  The
// counts equal those of testing every point (closed intervals; a NaN is inside no box).
__global__ void box_count_tiles_kernel(const float* __restrict__ sbox, const uint32_t* __restrict__ scnt,
                                       uint32_t stiles, const float* __restrict__ tbox,
                                       const float* __restrict__ pattrs, const uint32_t* __restrict__ tcnt,
                                       uint32_t tiles, uint32_t a, uint32_t a8, const float* __restrict__ lb,
                                       const float* __restrict__ rb, uint32_t qnum, uint32_t* __restrict__ box,
                                       uint32_t coarse) {
    const uint32_t lane = lane_id();
    const uint32_t q = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (q >= qnum) return;
    float lo[kMaxAttr], hi[kMaxAttr];
#pragma unroll
    for (uint32_t j = 0; j < kMaxAttr; ++j) {
        lo[j] = j < a ? lb[(size_t)q * a + j] : 0.0f;
        hi[j] = j < a ? rb[(size_t)q * a + j] : 0.0f;
    }
    uint32_t cnt = 0;
    for (uint32_t s0 = 0; s0 < stiles; s0 += 32) {
        const uint32_t st = s0 + lane;
        bool meet = false, inside = false;
        if (st < stiles) meet_inside(sbox + (size_t)st * 2 * a8, a, a8, lo, hi, meet, inside);
        if (inside) cnt += scnt[st];
        uint32_t ps = __ballot_sync(kFull, meet && !inside);
        while (ps) {
            const uint32_t ss = s0 + __ffs(ps) - 1;
            ps &= ps - 1;
            const uint32_t t = ss * kSuper + lane;
            bool tm = false, ti = false;
            if (t < tiles) meet_inside(tbox + (size_t)t * 2 * a8, a, a8, lo, hi, tm, ti);
            if (ti) cnt += tcnt[t];
            if (coarse) {  // estimate: half of each tile that meets the box without lying inside it
                if (tm && !ti) cnt += tcnt[t] >> 1;
                continue;
            }
            uint32_t pt = __ballot_sync(kFull, tm && !ti);
            while (pt) {
                const uint32_t tt = ss * kSuper + __ffs(pt) - 1;
                pt &= pt - 1;
                for (uint32_t r = lane; r < kBN; r += 32) {
                    const float* pa = pattrs + ((size_t)tt * kBN + r) * a;
                    bool ok = true;
#pragma unroll
                    for (uint32_t j = 0; j < kMaxAttr; ++j)
                        if (j < a) ok = ok & (pa[j] >= lo[j]) & (pa[j] <= hi[j]);
                    cnt += ok;
                }
            }
        }
    }
    for (int o = 16; o > 0; o >>= 1) cnt += __shfl_xor_sync(kFull, cnt, o);
    if (lane == 0) box[q] = cnt;
}
}  // namespace

void box_count_tiles(const DeviceIndex& d, const float* lb, const float* rb, uint32_t qnum, uint32_t* box,
                     cudaStream_t s, bool coarse) {
    box_count_tiles_kernel<<<(qnum + 7) / 8, 256, 0, s>>>(d.bf_sbox, d.bf_scnt, d.bf_stiles, d.bf_tbox, d.bf_attrs,
                                                          d.bf_tcnt, d.bf_tiles, d.a, tbox_stride(d.a), lb, rb, qnum,
                                                          box, coarse ? 1u : 0u);
}

bool bf_tc_usable(const DeviceIndex& d, uint32_t k) { return d.bf_ok && k >= 1 && k <= kMaxK; }

namespace {
// Working memory of one call, carved in this order from `base` (sizes only when base is NULL).
void carve_ws(const DeviceIndex& d, uint32_t qnum, uint32_t k, size_t tmp_sort, unsigned char* base, size_t* used,
              void** p) {
    const uint32_t qtiles = (qnum + kBM - 1) / kBM, qpad = qtiles * kBM, dp = d.bf_dp, a = d.a;
    const bool deep = k > kMaxKShallow;
    const size_t lists = deep ? Lists<true>::LISTS : Lists<false>::LISTS;
    const size_t km = deep ? Lists<true>::KM : Lists<false>::KM;
    Carve c{base};
    p[0] = c.take<unsigned long long>(qnum);  // keys
    p[1] = c.take<unsigned long long>(qnum);  // keys sorted
    p[2] = c.take<uint32_t>(qnum);            // iota
    p[3] = c.take<uint32_t>(qnum);            // sorted queries
    p[4] = c.take<unsigned char>(tmp_sort);
    p[5] = c.take<uint32_t>(qpad);            // perm
    p[6] = c.take<uint32_t>(qpad);            // flag
    p[7] = c.take<float>(qpad);               // pq
    p[8] = c.take<float>(qpad);               // dq
    p[9] = c.take<__half>((size_t)qpad * dp);
    p[10] = c.take<float>((size_t)qtiles * a);
    p[11] = c.take<float>((size_t)qtiles * a);
    p[12] = c.take<float>((size_t)qtiles * 4 * a);
    p[13] = c.take<float>((size_t)qtiles * 4 * a);
    p[14] = c.take<uint32_t>((size_t)qtiles * d.bf_tiles);
    p[15] = c.take<uint32_t>(qtiles);
    p[16] = c.take<uint2>((size_t)qpad * lists * km);
    p[17] = c.take<uint32_t>((size_t)qpad * lists + qpad);  // list counts, then row fallbacks
    p[18] = nullptr;
    p[19] = c.take<uint32_t>(qpad);            // published thresholds
    p[20] = c.take<uint32_t>(qtiles + 1 + 2);  // prefix of the tile counts, then W and G
    *used = c.used;
}

size_t sort_tmp_bytes(uint32_t qnum) {
    size_t tmp_sort = 0;
    cub::DeviceRadixSort::SortPairs(nullptr, tmp_sort, (unsigned long long*)nullptr, (unsigned long long*)nullptr,
                                    (uint32_t*)nullptr, (uint32_t*)nullptr, (int)qnum);
    return tmp_sort;
}
}  // namespace

size_t bf_tc_ws_bytes(const DeviceIndex& d, uint32_t qnum, uint32_t k) {
    void* P[21];
    size_t used = 0;
    carve_ws(d, qnum, k, sort_tmp_bytes(qnum), nullptr, &used, P);
    return used;
}

gf_status bf_tc_run(gf_index* idx, const float* queries, const float* lb, const float* rb, uint32_t qnum, uint32_t k,
                    uint32_t* ids, float* dist, void* ws, uint32_t* fb_list, uint32_t* fb_cnt, uint32_t test_every,
                    uint32_t test_wait, uint32_t* timeouts, uint32_t* products, cudaStream_t s,
                    const uint32_t* qmask) {
    DeviceIndex& d = idx->d;
    const uint32_t qtiles = (qnum + kBM - 1) / kBM, qpad = qtiles * kBM;
    const uint32_t dp = d.bf_dp, a = d.a;
    int nsm = 148;
    cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, d.device);
    const uint32_t grid = (uint32_t)std::max(1, nsm);  // persistent: one CTA per SM

    // list depth; stages of the chunk ring: as many as fit (at least 2); the query tile stays
    // in shared memory when it is at most kResidentDp wide and two stages still fit beside it
    const bool deep = k > kMaxKShallow;
    const uint32_t km = deep ? Lists<true>::KM : Lists<false>::KM, own = deep ? Lists<true>::OWN : Lists<false>::OWN;
    const uint32_t nlists = deep ? Lists<true>::LISTS : Lists<false>::LISTS;
    const uint32_t stream = (dp > kResidentDp || tc_layout(dp, 2, a, 0, km, own, kKC).total > kSmemLimit) ? 1u : 0u;
    // stage width: 64 elements, or 32 when 64-element stages would leave only two in the ring
    // and 32-element ones hold a fifth more useful bytes (measured on configuration 3, deep
    // lists at 96 dims: 3 stages of 64 against 6 of 32 made no difference, so 64 stays the
    // default; per-stage barrier work grows as the stages shrink)
    auto fit = [&](uint32_t kc, uint32_t max_stages) {
        uint32_t st = max_stages;
        while (st > 2 && tc_layout(dp, st, a, stream, km, own, kc).total > kSmemLimit) --st;
        return st;
    };
    auto in_flight = [&](uint32_t kc, uint32_t st) {  // useful bytes of st stages, averaged over a tile
        const uint32_t n = (dp + kc - 1) / kc;
        return (double)st * (double)dp * kBN * 2 / n;
    };
    uint32_t kc = kKC, stages = fit(kKC, 8);
    {
        const uint32_t st32 = fit(32, 16);
        if (stages <= 2 && in_flight(32, st32) > 1.2 * in_flight(kKC, stages)) {
            kc = 32;
            stages = st32;
        }
    }
    const uint32_t nck = (dp + kc - 1) / kc;
    const TcLayout Lo = tc_layout(dp, stages, a, stream, km, own, kc);
    if (Lo.total > kSmemLimit) return fail(GF_ERR_ARG, "tensor-core brute force: shared memory");

    size_t tmp_sort = sort_tmp_bytes(qnum);
    void* P[21];
    size_t used = 0;
    carve_ws(d, qnum, k, tmp_sort, static_cast<unsigned char*>(ws), &used, P);
    unsigned long long *keys = (unsigned long long*)P[0], *keys2 = (unsigned long long*)P[1];
    uint32_t *iota = (uint32_t*)P[2], *sorted = (uint32_t*)P[3];
    uint32_t *perm = (uint32_t*)P[5], *flag = (uint32_t*)P[6];
    float *pq = (float*)P[7], *dq = (float*)P[8];
    __half* at = (__half*)P[9];
    float *tq_lo = (float*)P[10], *tq_hi = (float*)P[11], *g_lo = (float*)P[12], *g_hi = (float*)P[13];
    uint32_t *tl = (uint32_t*)P[14], *tl_cnt = (uint32_t*)P[15];
    uint2* cand = (uint2*)P[16];
    uint32_t* cand_n = (uint32_t*)P[17];
    uint32_t* row_fb = cand_n + (size_t)qpad * nlists;
    uint32_t* thr_g = (uint32_t*)P[19];
    uint32_t* pre = (uint32_t*)P[20];
    uint32_t* sched = pre + qtiles + 1;

    gf_status st = GF_OK;
    auto ck = [&](cudaError_t e, const char* what) {
        if (e != cudaSuccess && st == GF_OK) st = cuda_fail(e, what);
    };
    ck(cudaMemsetAsync(cand_n, 0, sizeof(uint32_t) * ((size_t)qpad * nlists + qpad), s), "bf lists");
    bf_morton_kernel<<<(qnum + 255) / 256, 256, 0, s>>>(lb, rb, qnum, a, d.bf_arange, d.bf_arange + a, qmask, keys,
                                                         iota);
    ck(cub::DeviceRadixSort::SortPairs(P[4], tmp_sort, keys, keys2, iota, sorted, (int)qnum, 0, 64, s), "bf sort");
    const double omk = 1.0 - kappa_of(dp);
    bf_prep_kernel<<<(qpad + 7) / 8, 256, 0, s>>>(queries, qnum, d.dim, dp, sorted, qmask, qpad, d.bf_mean,
                                                  d.bf_scale, omk, perm, at, pq, dq, flag, thr_g);
    bf_boxes_kernel<<<qtiles, kBM, 0, s>>>(lb, rb, a, perm, flag, tq_lo, tq_hi, g_lo, g_hi);
    bf_tiles_kernel<<<qtiles, 256, 0, s>>>(d.bf_tbox, tbox_stride(a), d.bf_tiles, a, tq_lo, tq_hi, tl, tl_cnt, products);
    bf_sched_kernel<<<1, 32, 0, s>>>(tl_cnt, qtiles, grid, pre, sched);
    TcArgs T;
    T.at = at;
    T.xt = reinterpret_cast<const __half*>(d.bf_x);
    T.px = d.bf_px;
    T.pattrs = d.bf_attrs;
    T.rowpos = d.bf_rowpos;
    T.thr_g = thr_g;
    T.tbox = d.bf_tbox;
    T.a8 = tbox_stride(a);
    T.glo = g_lo;
    T.ghi = g_hi;
    T.lb = lb;
    T.rb = rb;
    T.perm = perm;
    T.flag = flag;
    T.tl = tl;
    T.pre = pre;
    T.sched = sched;
    T.row_fb = row_fb;
    T.qtiles = qtiles;
    T.polls = test_wait ? test_wait : kPolls;
    T.extra_tx = test_wait ? 16u : 0u;
    T.cand = cand;
    T.cand_n = cand_n;
    T.timeouts = timeouts;
    T.tiles = d.bf_tiles;
    T.a = a;
    T.dp = dp;
    T.nck = nck;
    T.kc = kc;
    T.stages = stages;
    T.stream_a = stream;
    void (*kern)(TcArgs) =
        deep ? (a == 1 ? bf_tc_kernel<1, true> : a == 2 ? bf_tc_kernel<2, true> : a == 3 ? bf_tc_kernel<3, true>
                : a == 4 ? bf_tc_kernel<4, true> : bf_tc_kernel<0, true>)
             : (a == 1 ? bf_tc_kernel<1, false> : a == 2 ? bf_tc_kernel<2, false> : a == 3 ? bf_tc_kernel<3, false>
                : a == 4 ? bf_tc_kernel<4, false> : bf_tc_kernel<0, false>);
    ck(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Lo.total), "bf smem");
    kern<<<grid, deep ? Lists<true>::THREADS : Lists<false>::THREADS, Lo.total, s>>>(T);
    MergeArgs M;
    M.cand = cand;
    M.cand_n = cand_n;
    M.perm = perm;
    M.flag = flag;
    M.pq = pq;
    M.dq = dq;
    M.queries = queries;
    M.vec32 = d.vec32;
    M.i2g = d.i2g;
    M.ids = ids;
    M.dists = dist;
    M.fb_list = fb_list;
    M.fb_cnt = fb_cnt;
    M.qpad = qpad;
    M.dim = d.dim;
    M.nch = d.d4 / 4;
    M.row_fb = row_fb;
    M.k = k;
    M.test_every = test_every;
    M.inv_s = 1.0f / d.bf_scale;
    M.dmax = d.bf_dmax;
    M.eta = (d.d4 / 8.0 + 16.0) * 0x1p-23;
    const size_t msmem = sizeof(float) * 8 * d.d4;
    if (deep)
        bf_merge_kernel<true><<<(qpad + 7) / 8, 256, msmem, s>>>(M);
    else
        bf_merge_kernel<false><<<(qpad + 7) / 8, 256, msmem, s>>>(M);
    ck(cudaGetLastError(), "bf kernels");
    return st;
}

}  // namespace gf
