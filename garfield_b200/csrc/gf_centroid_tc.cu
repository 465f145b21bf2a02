// Four nearest centroids per query on the tensor cores (dis_cal_tensor_core +
// select_topk_by_reduce_min, tools.cuh:1399-1537, which use WMMA on fp16 copies).
//
// Step 1, centroid_dot_tc_kernel: S = Q' C'^T with tcgen05.mma kind::tf32, where Q' and C'
// are the queries and centroids minus the centroids' mean m (centring shrinks the norms that
// the error bound below scales with).  Each operand value v is split into v_hi (v with its
// 13 low mantissa bits cleared, exact in tf32) and v_lo = v - v_hi, and every K step issues
// three MMAs, hi*hi + hi*lo + lo*hi, so the products carry ~21 significant bits instead of
// tf32's 11.  One CTA computes 128 queries x 128 centroids with fp32 accumulation in 128
// TMEM columns; operands are staged K-major in shared memory 16 dimensions at a time in
// the no-swizzle core-matrix layout (8 rows x 16 bytes per core matrix; LBO = distance of
// the next 16-byte column of core matrices, SBO = distance of the next 8 rows).  The next
// chunk is loaded into registers while the MMAs of the current one run; one thread issues
// the MMAs and commits them to an mbarrier; after the last chunk each warp reads its 32 TMEM
// lanes (= 32 query rows) with tcgen05.ld, transposes 32 x 32 blocks through shared memory
// and writes S with one 128-byte row segment per store instruction.
//
// Step 2, centroid_select_kernel (one warp per query): the distances
//   d~ = (|q'|^2 + |c'|^2) - 2 S
// are only approximate; the canonical distance (one sequential fp32 fma chain over the
// dimensions of the uncentred vectors, oracle orc_dist_seq) lies within [lb, ub] of d~ by an
// error bound covering the split products (relative 3 * 2^-20 each), fp32 accumulation in
// any order with truncation, the centring's roundings, the norms, the epilogue's own
// roundings and the canonical chain's rounding.  With U the 4th smallest ub, every centroid
// whose lb is above U is provably outside the 4 nearest; the others are re-ranked with the
// exact canonical distance (candidate rows staged through shared memory with coalesced
// loads, one candidate per lane), ties by centroid id.  A NaN distance ranks after every
// number (the device key order): a NaN centroid (the 0/0 centroid of an empty cluster)
// never lowers U and is left out while 4 candidates with numbers remain.  The result is
// bit-identical to the CUDA-core kernel whatever the data; when more than kMaxCand
// centroids survive the bound, fewer than 4 remain, or the query is not finite, a query
// re-ranks every centroid instead.
#include <cstdint>

#include "gf_device.cuh"
#include "gf_internal.h"

namespace gf {
namespace {

using namespace dev;

constexpr uint32_t kTcM = 128, kTcN = 128, kTcKC = 16;  // tile rows, columns, K chunk (elements)
constexpr uint32_t kTcChunkFloats = kTcM * kTcKC;        // one operand part of one chunk
constexpr uint32_t kTcSmem = 55 * 1024;  // dynamic shared memory per CTA (32 KB used): caps
                                         // residency at 4 CTAs per SM = 4 x 128 TMEM columns
constexpr uint32_t kTcWaitPolls = 1u << 20;
constexpr uint32_t kMaxCand = 128;
static_assert(kTcM == kTcN, "the staging maps one thread layout onto both operands");

// Shared-memory matrix descriptor, K-major, no swizzle (version 1 for sm_100).
__device__ __forceinline__ uint64_t kmajor_desc(const void* p, uint32_t lbo, uint32_t sbo) {
    uint64_t d = (uint64_t)((smem_u32(p) >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;
    return d;
}

// Instruction descriptor: D f32, A and B tf32, both K-major, N = kTcN, M = kTcM.
constexpr uint32_t kIdesc = (1u << 4) | (2u << 7) | (2u << 10) | ((kTcN >> 3) << 17) | ((kTcM >> 4) << 24);

__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void mma_tf32(uint32_t tmem, uint64_t ad, uint64_t bd, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem),
        "l"(ad), "l"(bd), "r"(kIdesc), "r"(acc), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
}

// Float index of element (r, 4j) of a 128 x kTcKC chunk in the core-matrix layout: 16-byte
// column j holds 16 consecutive 128-byte core matrices (LBO = 2048 B, SBO = 128 B).
__device__ __forceinline__ uint32_t cm_index(uint32_t r, uint32_t j) {
    return ((j * (kTcM / 8) + (r >> 3)) * 8 + (r & 7)) * 4;
}

// Four centred values v[k..k+3] - m[k..k+3] of row `row` (zeros past the matrix).
__device__ __forceinline__ float4 load_centred(const float* __restrict__ src, uint32_t row, uint32_t nrows,
                                               uint32_t dim, uint32_t k, float4 m) {
    float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (row >= nrows || k >= dim) return v;
    const float* p = src + (size_t)row * dim + k;
    if ((dim & 3u) == 0) {
        v = __ldg(reinterpret_cast<const float4*>(p));
    } else {
        v.x = p[0];
        if (k + 1 < dim) v.y = p[1];
        if (k + 2 < dim) v.z = p[2];
        if (k + 3 < dim) v.w = p[3];
    }
    v.x = k < dim ? __fsub_rn(v.x, m.x) : 0.0f;
    v.y = k + 1 < dim ? __fsub_rn(v.y, m.y) : 0.0f;
    v.z = k + 2 < dim ? __fsub_rn(v.z, m.z) : 0.0f;
    v.w = k + 3 < dim ? __fsub_rn(v.w, m.w) : 0.0f;
    return v;
}

// 16 consecutive TMEM columns of this warp's 32 lanes (lane i gets row i).
__device__ __forceinline__ void tmem_ld16(uint32_t addr, uint32_t* v) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];\n"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
          "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(addr));
}

__device__ __forceinline__ float tf32_hi(float v) { return __uint_as_float(__float_as_uint(v) & 0xFFFFE000u); }

__device__ __forceinline__ void store_split(float* hi, float* lo, uint32_t at, float4 v) {
    const float4 h = make_float4(tf32_hi(v.x), tf32_hi(v.y), tf32_hi(v.z), tf32_hi(v.w));
    const float4 l = make_float4(__fsub_rn(v.x, h.x), __fsub_rn(v.y, h.y), __fsub_rn(v.z, h.z), __fsub_rn(v.w, h.w));
    *reinterpret_cast<float4*>(hi + at) = h;
    *reinterpret_cast<float4*>(lo + at) = l;
}

__global__ void __launch_bounds__(128) centroid_dot_tc_kernel(const float* __restrict__ Q, uint32_t qnum, uint32_t dim,
                                                              const float* __restrict__ Cm, uint32_t C,
                                                              const float* __restrict__ mean, float* __restrict__ S,
                                                              uint32_t s_stride, uint32_t* __restrict__ timeouts,
                                                              const uint32_t* __restrict__ live) {
    extern __shared__ __align__(128) unsigned char tc_smem[];
    float* Ah = reinterpret_cast<float*>(tc_smem);  // queries, hi parts
    float* Al = Ah + kTcChunkFloats;                // queries, lo parts
    float* Bh = Al + kTcChunkFloats;                // centroids, hi parts
    float* Bl = Bh + kTcChunkFloats;                // centroids, lo parts
    __shared__ __align__(8) uint64_t bar;
    __shared__ uint32_t tmem_base;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t q0 = blockIdx.x * kTcM, c0 = blockIdx.y * kTcN;
    if (live) qnum = min(live[0], qnum);  // rows in use (a shard's listed queries)
    if (q0 >= qnum) return;               // before the TMEM allocation: the whole block leaves
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base)),
                     "r"(kTcN));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
    }
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base;
    // staging map: a warp covers 8 rows x 4 16-byte columns per step (16 sectors per load,
    // 4 shared-memory wavefronts per store); thread t takes rows (t/32 + 4 it) * 8 + t % 8
    const uint32_t jcol = (threadIdx.x >> 3) & 3u, rlo = threadIdx.x & 7u, rgrp = threadIdx.x >> 5;
    float4 ra[4], rb[4];
    auto load = [&](uint32_t k0) {
        const uint32_t k = k0 + jcol * 4;
        float4 m = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (k < dim) {
            m.x = mean[k];
            if (k + 1 < dim) m.y = mean[k + 1];
            if (k + 2 < dim) m.z = mean[k + 2];
            if (k + 3 < dim) m.w = mean[k + 3];
        }
#pragma unroll
        for (uint32_t it = 0; it < 4; ++it) {
            const uint32_t r = (rgrp + 4 * it) * 8 + rlo;
            ra[it] = load_centred(Q, q0 + r, qnum, dim, k, m);
            rb[it] = load_centred(Cm, c0 + r, C, dim, k, m);
        }
    };
    load(0);
    uint32_t phase = 0;
    bool ok = true;
    for (uint32_t k0 = 0; k0 < dim; k0 += kTcKC) {
#pragma unroll
        for (uint32_t it = 0; it < 4; ++it) {
            const uint32_t at = cm_index((rgrp + 4 * it) * 8 + rlo, jcol);
            store_split(Ah, Al, at, ra[it]);
            store_split(Bh, Bl, at, rb[it]);
        }
        fence_proxy_async_smem();  // the operand writes become visible to the tensor cores
        __syncthreads();
        if (threadIdx.x == 0) {
            tc_fence_after();
#pragma unroll
            for (uint32_t s = 0; s < kTcKC / 8; ++s) {  // K = 8 per MMA: two 16-byte columns
                const uint32_t off = s * 2 * kTcM * 4;
                const uint64_t ah = kmajor_desc(Ah + off, kTcM * 16, 128), al = kmajor_desc(Al + off, kTcM * 16, 128);
                const uint64_t bh = kmajor_desc(Bh + off, kTcN * 16, 128), bl = kmajor_desc(Bl + off, kTcN * 16, 128);
                mma_tf32(tmem, ah, bh, (k0 > 0 || s > 0) ? 1u : 0u);
                mma_tf32(tmem, ah, bl, 1u);
                mma_tf32(tmem, al, bh, 1u);
            }
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                             smem_u32(&bar))
                         : "memory");
        }
        if (k0 + kTcKC < dim) load(k0 + kTcKC);  // overlaps the MMAs
        // the MMAs must finish reading shared memory before the next chunk overwrites it
        uint32_t polls = 0;
        bool done;
        while (!(done = mbar_try_wait(&bar, phase, 1000)) && ++polls < kTcWaitPolls) {
        }
        ok = __syncthreads_and(done);
        if (!ok) break;
        phase ^= 1u;
    }
    tc_fence_after();
    if (ok) {
        // TMEM -> registers (row = lane) -> shared memory (32 x 32, padded) -> S, one
        // 128-byte row segment per store instruction; the operand buffers are free now
        float* stg = reinterpret_cast<float*>(tc_smem) + warp * 32 * 33;
        const uint32_t taddr = tmem + ((warp * 32u) << 16);
        for (uint32_t cb = 0; cb < kTcN; cb += 32) {
            uint32_t v[32];
            tmem_ld16(taddr + cb, v);
            tmem_ld16(taddr + cb + 16, v + 16);
            // the wait names the loaded registers so that no use of them is scheduled before it
            asm volatile("tcgen05.wait::ld.sync.aligned;"
                         : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]), "+r"(v[6]),
                           "+r"(v[7]), "+r"(v[8]), "+r"(v[9]), "+r"(v[10]), "+r"(v[11]), "+r"(v[12]), "+r"(v[13]),
                           "+r"(v[14]), "+r"(v[15]), "+r"(v[16]), "+r"(v[17]), "+r"(v[18]), "+r"(v[19]), "+r"(v[20]),
                           "+r"(v[21]), "+r"(v[22]), "+r"(v[23]), "+r"(v[24]), "+r"(v[25]), "+r"(v[26]), "+r"(v[27]),
                           "+r"(v[28]), "+r"(v[29]), "+r"(v[30]), "+r"(v[31])
                         :
                         : "memory");
#pragma unroll
            for (uint32_t j = 0; j < 32; ++j) stg[lane * 33 + j] = __uint_as_float(v[j]);
            __syncwarp();
            for (uint32_t r = 0; r < 32; ++r) {
                const uint32_t q = q0 + warp * 32 + r;
                if (q < qnum) S[(size_t)q * s_stride + c0 + cb + lane] = stg[r * 33 + lane];
            }
            __syncwarp();
        }
    } else if (threadIdx.x == 0) {
        atomicAdd(timeouts, 1u);
        // the MMAs may still be running: wait for them (again bounded) before freeing TMEM
        uint32_t polls = 0;
        while (!mbar_try_wait(&bar, phase, 1000) && ++polls < kTcWaitPolls) {
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTcN));
}

// Sorted 4-list of 64-bit keys: insert one key.
__device__ __forceinline__ void top4_insert(key_t* t, key_t k) {
    if (k >= t[3]) return;
    t[3] = k;
#pragma unroll
    for (int r = 3; r > 0; --r)
        if (t[r] < t[r - 1]) {
            const key_t x = t[r];
            t[r] = t[r - 1];
            t[r - 1] = x;
        }
}

// Warp-wide merge of the lanes' sorted 4-lists (butterfly): every lane ends with the 4
// smallest keys of the warp.
__device__ __forceinline__ void top4_warp(key_t* t) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        key_t other[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) other[r] = __shfl_xor_sync(kFull, t[r], o);
#pragma unroll
        for (int r = 0; r < 4; ++r) top4_insert(t, other[r]);
    }
}

// Exact re-rank staging: up to 32 candidate rows and the query, kRrDims dimensions at a
// time, in shared memory (row stride kRrStride floats: lane i reading row i with 16-byte
// loads takes the minimum 4 wavefronts per instruction).
constexpr uint32_t kRrDims = 64;
constexpr uint32_t kRrStride = kRrDims + 4;
constexpr uint32_t kRrWarpFloats = 33 * kRrStride;       // 32 candidates + the query
constexpr uint32_t kSelectSmem = 4 * kRrWarpFloats * 4;  // bytes per 4-warp block

__device__ __forceinline__ void chain4(float& acc, float4 q, float4 x) {
    float df = __fsub_rn(q.x, x.x);
    acc = __fmaf_rn(df, df, acc);
    df = __fsub_rn(q.y, x.y);
    acc = __fmaf_rn(df, df, acc);
    df = __fsub_rn(q.z, x.z);
    acc = __fmaf_rn(df, df, acc);
    df = __fsub_rn(q.w, x.w);
    acc = __fmaf_rn(df, df, acc);
}

// Canonical distances (oracle orc_dist_seq: one fma chain over d = 0..dim-1) of query q to
// the ng <= 32 centroids id(0..ng-1); lane i returns candidate i's (lanes >= ng: garbage).
// Rows with dim % 4 == 0 are staged by the whole warp, half a warp per 64-dimension row
// segment (16-byte loads, 8 in flight per lane), then each lane runs its own chain from
// shared memory; other rows are read directly.  Every lane of the warp calls this together.
template <class Id>
__device__ __forceinline__ float chain_dists(const float* __restrict__ q, const float* __restrict__ Cm, uint32_t dim,
                                            uint32_t ng, Id id, float* ws, uint32_t lane) {
    float acc = 0.0f;
    if ((dim & 3u) != 0) {
        const float* x = Cm + (size_t)id(min(lane, ng - 1)) * dim;
        for (uint32_t d = 0; d < dim; ++d) {
            const float df = __fsub_rn(q[d], x[d]);
            acc = __fmaf_rn(df, df, acc);
        }
        return acc;
    }
    const uint32_t half = lane >> 4, hl = lane & 15u;
    float* qs = ws + 32 * kRrStride;
    for (uint32_t k0 = 0; k0 < dim; k0 += kRrDims) {
        const uint32_t n4 = min(kRrDims, dim - k0) >> 2, k = k0 + 4 * hl;
        for (uint32_t i0 = 0; i0 < ng; i0 += 16) {  // 8 loads per lane = 16 rows per batch
            float4 v[8];
#pragma unroll
            for (uint32_t t = 0; t < 8; ++t) {
                const uint32_t i = i0 + 2 * t + half;
                if (i < ng && hl < n4) v[t] = __ldg(reinterpret_cast<const float4*>(Cm + (size_t)id(i) * dim + k));
            }
#pragma unroll
            for (uint32_t t = 0; t < 8; ++t) {
                const uint32_t i = i0 + 2 * t + half;
                if (i < ng && hl < n4) *reinterpret_cast<float4*>(ws + i * kRrStride + 4 * hl) = v[t];
            }
        }
        if (half == 0 && hl < n4) *reinterpret_cast<float4*>(qs + 4 * hl) = __ldg(reinterpret_cast<const float4*>(q + k));
        __syncwarp();
        const float* mine = ws + lane * kRrStride;
#pragma unroll 4
        for (uint32_t t = 0; t < n4; ++t)
            chain4(acc, *reinterpret_cast<const float4*>(qs + 4 * t), *reinterpret_cast<const float4*>(mine + 4 * t));
        __syncwarp();  // before the next segment overwrites the staging area
    }
    return acc;
}

// Error-bound constants of one query (see the file comment).  For a centroid with centred
// squared norm cn (norm ncn) and approximate distance dt, |canonical - dt| stays within
//   E = k_prod ncn + k_norm (qn + cn) + k_cent (nq + ncn)^2 + k_dt |dt|
// (products, norms and their sum, centring, the subtraction forming dt) before the
// canonical chain's own relative error g_can.  With (nq + ncn)^2 <= 2 (qn + cn) and
// |dt| <= (2 + 2 a_inner)(qn + cn) this is at most  B ncn + D (qn + cn).
struct Bound {
    float B, D, up, dn;
};

__device__ __forceinline__ Bound make_bound(float qn, uint32_t dim) {
    const float u = 5.9604645e-8f;  // 2^-24
    const float gD = (float)(dim + 1) * u * 1.0001f;
    // |S - q'.c'| <= a_inner |q'| |c'|: the split products (3 * 2^-20 relative each) and the
    // fp32 accumulation of 3 * dim products, its term doubled in case the tensor cores
    // truncate instead of rounding
    const float a_inner = 3.01f * 9.5367432e-7f + 2.0f * (float)(3 * dim + 2) * u * 1.003f;
    const float s = 1.05f;                    // slack for the roundings of the bound's own arithmetic
    const float k_prod = 2.0f * a_inner * sqrtf(qn);  // 2 S
    const float k_norm = gD + 2.0f * u;       // both squared norms and the sum qn + cn
    const float k_cent = 2.1f * u;            // rounding of the centring subtractions
    const float k_dt = 2.0f * u;              // the subtraction forming dt
    const float g_can = gD + 2.0f * u;        // the canonical chain against the exact distance
    Bound b;
    b.B = s * k_prod;
    b.D = s * (k_norm + 2.0f * k_cent + (2.0f + 2.0f * a_inner) * k_dt);
    b.up = (1.0f + g_can) * (1.0f + 4.0f * u);
    b.dn = (1.0f - g_can) * (1.0f - 4.0f * u);
    return b;
}

__global__ void __launch_bounds__(128) centroid_select_kernel(const float* __restrict__ S, uint32_t s_stride,
                                                              uint32_t qnum, uint32_t C,
                                                              const float* __restrict__ Q, uint32_t dim,
                                                              const float* __restrict__ Cm,
                                                              const float* __restrict__ mean,
                                                              const float2* __restrict__ cnorm,
                                                              uint32_t* __restrict__ top4,
                                                              uint32_t* __restrict__ counters,
                                                              const uint32_t* __restrict__ live) {
    __shared__ uint32_t cand[4][kMaxCand];
    extern __shared__ __align__(16) float rr_smem[];  // kSelectSmem bytes
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t q = blockIdx.x * 4 + warp;
    if (live) qnum = min(live[0], qnum);  // row q is query live[1 + q]
    if (q >= qnum) return;
    const float kInf = __int_as_float(0x7f800000);
    const float* qv = Q + (size_t)q * dim;
    float qn = 0.0f;  // centred squared norm
    for (uint32_t d = lane; d < dim; d += 32) {
        const float t = __fsub_rn(qv[d], mean[d]);
        qn = __fmaf_rn(t, t, qn);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) qn = __fadd_rn(qn, __shfl_xor_sync(kFull, qn, o));
    const Bound b = make_bound(qn, dim);
    const float* Sq = S + (size_t)q * s_stride;
    float* ws = rr_smem + warp * kRrWarpFloats;
    // pass 1: every lane keeps its 4 smallest upper bounds; lower bounds are stashed in the
    // warp's staging area when they fit (a NaN centroid's as +inf: it is kept only when
    // U = +inf, i.e. when fewer than 4 centroids have numbers)
    const bool stash = C <= kRrWarpFloats;
    float t0 = kInf, t1 = kInf, t2 = kInf, t3 = kInf;
    for (uint32_t c = lane; c < C; c += 32) {
        const float2 cn = cnorm[c];
        const float qc = qn + cn.x;
        const float dt = __fmaf_rn(-2.0f, Sq[c], qc);
        const float E = __fmaf_rn(b.B, cn.y, b.D * qc);
        float ub = (dt + E) * b.up;
        ub = ub >= 0.0f ? ub : (ub < 0.0f ? 0.0f : kInf);  // NaN bounds nothing: +inf
        if (stash) ws[c] = isnan(cn.x) ? kInf : (dt - E) * b.dn;
        if (ub < t3) {
            t3 = ub;
            if (t3 < t2) { const float x = t2; t2 = t3; t3 = x; }
            if (t2 < t1) { const float x = t1; t1 = t2; t2 = x; }
            if (t1 < t0) { const float x = t0; t0 = t1; t1 = x; }
        }
    }
    // U = 4th smallest over the warp: four rounds of popping the warp minimum (the bounds
    // are >= +0, so their bit patterns order like the values)
    uint32_t Ub = 0;
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        Ub = __reduce_min_sync(kFull, __float_as_uint(t0));
        const uint32_t win = __ffs(__ballot_sync(kFull, __float_as_uint(t0) == Ub)) - 1;
        if (lane == win) {
            t0 = t1;
            t1 = t2;
            t2 = t3;
            t3 = kInf;
        }
    }
    const float U = __uint_as_float(Ub);
    __syncwarp();
    // pass 2: candidates whose lower bound does not exceed U (a NaN bound is kept)
    uint32_t nc = 0;
    for (uint32_t c0 = 0; c0 < C; c0 += 32) {
        const uint32_t c = c0 + lane;
        bool keep = false;
        if (c < C) {
            float lb;
            if (stash) {
                lb = ws[c];
            } else {
                const float2 cn = cnorm[c];
                const float qc = qn + cn.x;
                const float dt = __fmaf_rn(-2.0f, Sq[c], qc);
                lb = isnan(cn.x) ? kInf : (dt - __fmaf_rn(b.B, cn.y, b.D * qc)) * b.dn;
            }
            keep = !(lb > U);
        }
        const uint32_t m = __ballot_sync(kFull, keep);
        const uint32_t at = nc + __popc(m & lanemask_lt());
        if (keep && at < kMaxCand) cand[warp][at] = c;
        nc += __popc(m);
    }
    __syncwarp();
    // re-rank every centroid when the bound kept too many, when fewer than 4 candidates
    // remain or when the query is not finite
    const bool scan_all = nc > kMaxCand || nc < 4 || !(fabsf(qn) < kInf);
    if (lane == 0) {
        if (scan_all) atomicAdd(counters + 1, 1u);
        atomicAdd(counters + 2, scan_all ? C : nc);
    }
    const uint32_t n = scan_all ? C : nc;
    const uint32_t* cw = cand[warp];
    key_t mine;
    if (n <= 32) {  // one candidate per lane: four rounds of popping the warp's smallest key
        auto id = [&](uint32_t i) { return scan_all ? i : cw[i]; };
        const float acc = chain_dists(qv, Cm, dim, n, id, ws, lane);
        key_t k = lane < n ? make_key(acc, id(lane), 0) : kEmptyKey;
        mine = kEmptyKey;
#pragma unroll
        for (uint32_t r = 0; r < 4; ++r) {
            const uint32_t hi = (uint32_t)(k >> 32), lo = (uint32_t)k;
            const uint32_t mh = __reduce_min_sync(kFull, hi);
            const uint32_t ml = __reduce_min_sync(kFull, hi == mh ? lo : 0xFFFFFFFFu);
            if (lane == r) mine = ((key_t)mh << 32) | ml;
            if (hi == mh && lo == ml) k = kEmptyKey;
        }
    } else {  // 32 candidates at a time (lane i: candidate g0 + i), per-lane lists merged
        key_t best[4] = {kEmptyKey, kEmptyKey, kEmptyKey, kEmptyKey};
        for (uint32_t g0 = 0; g0 < n; g0 += 32) {
            const uint32_t ng = min(32u, n - g0);
            auto id = [&](uint32_t i) { return scan_all ? g0 + i : cw[g0 + i]; };
            const float acc = chain_dists(qv, Cm, dim, ng, id, ws, lane);
            if (lane < ng) top4_insert(best, make_key(acc, id(lane), 0));
        }
        top4_warp(best);
        mine = best[0];
#pragma unroll
        for (uint32_t r = 1; r < 4; ++r)
            if (lane == r) mine = best[r];
    }
    const size_t out = live ? live[1 + q] : q;
    if (lane < 4) top4[out * 4 + lane] = mine == kEmptyKey ? kEmpty : key_pos(mine);
}

}  // namespace

bool centroid_tc_usable(const DeviceIndex& d) { return d.C >= kTcN && d.cnorm != nullptr && d.cmean != nullptr; }

size_t centroid_tc_stride(const DeviceIndex& d) { return ((size_t)d.C + kTcN - 1) / kTcN * kTcN; }

gf_status centroid_top4_tc(const DeviceIndex& d, const float* q32, uint32_t qnum, float* S, uint32_t* top4,
                           uint32_t* counters, cudaStream_t s, const uint32_t* live) {
    static bool attr_set[64] = {false};
    if (d.device >= 0 && d.device < 64 && !attr_set[d.device]) {
        GF_CUDA(cudaFuncSetAttribute(centroid_dot_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)kTcSmem));
        GF_CUDA(cudaFuncSetAttribute(centroid_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)kSelectSmem));
        attr_set[d.device] = true;
    }
    const uint32_t stride = (uint32_t)centroid_tc_stride(d);
    dim3 grid((qnum + kTcM - 1) / kTcM, (d.C + kTcN - 1) / kTcN);
    centroid_dot_tc_kernel<<<grid, 128, kTcSmem, s>>>(q32, qnum, d.dim, d.centroids, d.C, d.cmean, S, stride,
                                                      counters, live);
    GF_CUDA(cudaGetLastError());
    centroid_select_kernel<<<(qnum + 3) / 4, 128, kSelectSmem, s>>>(S, stride, qnum, d.C, q32, d.dim, d.centroids, d.cmean,
                                                         reinterpret_cast<const float2*>(d.cnorm), top4, counters, live);
    GF_CUDA(cudaGetLastError());
    return GF_OK;
}

}  // namespace gf
