// Device helpers shared by the search and brute-force kernels: canonical distances,
// keys, warp-level sort/merge primitives and the visited hash.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include "gf_internal.h"

namespace gf {
namespace dev {

constexpr unsigned kFull = 0xFFFFFFFFu;

__device__ __forceinline__ uint32_t lane_id() { return threadIdx.x & 31u; }

__device__ __forceinline__ uint32_t lanemask_lt() {
    uint32_t m;
    asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
    return m;
}

// Sort key of a list entry: (distance bits, position); empty entries sort last.
// Distances are >= +0, so their bit patterns order like the values.
__device__ __forceinline__ uint64_t mkkey(float d, uint32_t w) {
    return ((uint64_t)__float_as_uint(d) << 32) | (w == kEmpty ? kEmpty : (w & kPosMask));
}

// Row chunks loaded per batch in dist16 (loads in flight per lane).
#ifndef GF_DIST_GROUP
#define GF_DIST_GROUP 8
#endif
constexpr int kDistGroup = GF_DIST_GROUP;

// 16-byte read-only load of a stored row chunk.
__device__ __forceinline__ uint4 ldg16(const uint4* p) { return __ldg(p); }

// Canonical fp16 squared distance (same order as the oracle's orc_dist16): sixteen
// partials, partial u takes chunks u, u+16, ... (8 halves each) with one fused
// multiply-add per element on fp32 differences, then the pairwise tree 8/4/2/1.
// qs: the query as fp32 (converted from its fp16 row), nch = row chunks.
__device__ __forceinline__ float dist16(const uint4* __restrict__ row, const float* __restrict__ qs, uint32_t nch) {
    float p[16];
#pragma unroll
    for (int u = 0; u < 16; ++u) p[u] = 0.0f;
    for (uint32_t c0 = 0; c0 < nch; c0 += 16) {
#pragma unroll
        for (int h = 0; h < 16; h += kDistGroup) {
        uint4 x[kDistGroup];
#pragma unroll
        for (int v = 0; v < kDistGroup; ++v)
            if (c0 + h + v < nch) x[v] = ldg16(row + c0 + h + v);
#pragma unroll
        for (int v = 0; v < kDistGroup; ++v) {
            const int u = h + v;
            if (c0 + u < nch) {
                const float4 qa = *reinterpret_cast<const float4*>(qs + (c0 + u) * 8);
                const float4 qb = *reinterpret_cast<const float4*>(qs + (c0 + u) * 8 + 4);
                const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&x[v].x));
                const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&x[v].y));
                const float2 f2 = __half22float2(*reinterpret_cast<const __half2*>(&x[v].z));
                const float2 f3 = __half22float2(*reinterpret_cast<const __half2*>(&x[v].w));
                float acc = p[u], t;
                t = __fsub_rn(qa.x, f0.x); acc = __fmaf_rn(t, t, acc);
                t = __fsub_rn(qa.y, f0.y); acc = __fmaf_rn(t, t, acc);
                t = __fsub_rn(qa.z, f1.x); acc = __fmaf_rn(t, t, acc);
                t = __fsub_rn(qa.w, f1.y); acc = __fmaf_rn(t, t, acc);
                t = __fsub_rn(qb.x, f2.x); acc = __fmaf_rn(t, t, acc);
                t = __fsub_rn(qb.y, f2.y); acc = __fmaf_rn(t, t, acc);
                t = __fsub_rn(qb.z, f3.x); acc = __fmaf_rn(t, t, acc);
                t = __fsub_rn(qb.w, f3.y); acc = __fmaf_rn(t, t, acc);
                p[u] = acc;
            }
        }
        }
    }
#pragma unroll
    for (int s = 8; s >= 1; s >>= 1)
#pragma unroll
        for (int i = 0; i < s; ++i) p[i] = __fadd_rn(p[i], p[i + s]);
    return p[0];
}

// Canonical fp16 distance of a row staged in shared memory (nch chunks of 8 halves,
// row stride a multiple of 16 chunks).  Lane r reads chunk c0 + ((c + r) & 15) at step c,
// so the 8 lanes of a shared-memory phase touch 8 different 16-byte bank groups.
// Partial c of this lane then holds canonical partial (c + r) & 15; the pairwise tree
// pairs indices that differ in one bit (i, i ^ s), a pairing that rotation by r maps
// onto itself, and fp32 addition is commutative, so the result equals dist16 / the
// oracle's orc_dist16 bit for bit.  qa/qb: the query's first/second 4 floats of each chunk.
__device__ __forceinline__ float dist16_staged(const uint4* srow, const float4* qa, const float4* qb, uint32_t nch,
                                               uint32_t rot) {
    float p[16];
#pragma unroll
    for (int u = 0; u < 16; ++u) p[u] = 0.0f;
    for (uint32_t c0 = 0; c0 < nch; c0 += 16) {
#pragma unroll
        for (int c = 0; c < 16; ++c) {
            const uint32_t u = c0 + ((c + rot) & 15u);
            if (u < nch) {
                const uint4 x = srow[u];
                const float4 a = qa[u];
                const float4 b = qb[u];
                const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&x.x));
                const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&x.y));
                const float2 f2 = __half22float2(*reinterpret_cast<const __half2*>(&x.z));
                const float2 f3 = __half22float2(*reinterpret_cast<const __half2*>(&x.w));
                float acc = p[c], t;
                t = __fsub_rn(a.x, f0.x); acc = __fmaf_rn(t, t, acc);
                t = __fsub_rn(a.y, f0.y); acc = __fmaf_rn(t, t, acc);
                t = __fsub_rn(a.z, f1.x); acc = __fmaf_rn(t, t, acc);
                t = __fsub_rn(a.w, f1.y); acc = __fmaf_rn(t, t, acc);
                t = __fsub_rn(b.x, f2.x); acc = __fmaf_rn(t, t, acc);
                t = __fsub_rn(b.y, f2.y); acc = __fmaf_rn(t, t, acc);
                t = __fsub_rn(b.z, f3.x); acc = __fmaf_rn(t, t, acc);
                t = __fsub_rn(b.w, f3.y); acc = __fmaf_rn(t, t, acc);
                p[c] = acc;
            }
        }
    }
#pragma unroll
    for (int s = 8; s >= 1; s >>= 1)
#pragma unroll
        for (int i = 0; i < s; ++i) p[i] = __fadd_rn(p[i], p[i + s]);
    return p[0];
}

// 16-byte asynchronous global -> shared copy (cp.async, L2 only) and its fences.
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
    uint32_t d = (uint32_t)__cvta_generic_to_shared(smem_dst);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(d), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;\n" ::: "memory");
}

// Canonical fp32 squared distance (oracle orc_dist32): chunks of 4 floats.
__device__ __forceinline__ float dist32(const float4* __restrict__ row, const float4* __restrict__ q, uint32_t nch) {
    float p[16];
#pragma unroll
    for (int u = 0; u < 16; ++u) p[u] = 0.0f;
    for (uint32_t c0 = 0; c0 < nch; c0 += 16) {
        float4 x[16];
#pragma unroll
        for (int u = 0; u < 16; ++u)
            if (c0 + u < nch) x[u] = __ldg(row + c0 + u);
#pragma unroll
        for (int u = 0; u < 16; ++u) {
            if (c0 + u < nch) {
                const float4 qv = q[c0 + u];
                float acc = p[u], t;
                t = __fsub_rn(qv.x, x[u].x); acc = __fmaf_rn(t, t, acc);
                t = __fsub_rn(qv.y, x[u].y); acc = __fmaf_rn(t, t, acc);
                t = __fsub_rn(qv.z, x[u].z); acc = __fmaf_rn(t, t, acc);
                t = __fsub_rn(qv.w, x[u].w); acc = __fmaf_rn(t, t, acc);
                p[u] = acc;
            }
        }
    }
#pragma unroll
    for (int s = 8; s >= 1; s >>= 1)
#pragma unroll
        for (int i = 0; i < s; ++i) p[i] = __fadd_rn(p[i], p[i + s]);
    return p[0];
}

// Closed-box test of one point (merge_top_with_recycle_list's filter, gpu_graph.cu:514-520).
__device__ __forceinline__ bool in_box(const float* __restrict__ attrs, uint32_t pos, uint32_t a,
                                       const float* __restrict__ lb, const float* __restrict__ rb) {
    bool ok = true;
    for (uint32_t j = 0; j < a; ++j) {
        float v = __ldg(attrs + (size_t)pos * a + j);
        ok = ok && (v >= lb[j]) && (v <= rb[j]);
    }
    return ok;
}

// Warp bitonic sort of (d, w) pairs in shared memory by mkkey; n is a power of two.
__device__ __forceinline__ void warp_sort(float* d, uint32_t* w, uint32_t n) {
    const uint32_t lane = lane_id();
    for (uint32_t k = 2; k <= n; k <<= 1) {
        for (uint32_t j = k >> 1; j > 0; j >>= 1) {
            for (uint32_t i = lane; i < (n >> 1); i += 32) {
                uint32_t lo = 2 * j * (i / j) + (i % j);
                uint32_t hi = lo + j;
                bool asc = (lo & k) == 0;
                float dl = d[lo], dh = d[hi];
                uint32_t wl = w[lo], wh = w[hi];
                if ((mkkey(dl, wl) > mkkey(dh, wh)) == asc) {
                    d[lo] = dh;
                    d[hi] = dl;
                    w[lo] = wh;
                    w[hi] = wl;
                }
            }
            __syncwarp();
        }
    }
}

// Number of entries of the sorted list (d, w)[0..n) whose key is below `key`.
__device__ __forceinline__ uint32_t count_below(const float* d, const uint32_t* w, uint32_t n, uint64_t key) {
    uint32_t lo = 0, hi = n;
    while (lo < hi) {
        uint32_t mid = (lo + hi) >> 1;
        if (mkkey(d[mid], w[mid]) < key)
            lo = mid + 1;
        else
            hi = mid;
    }
    return lo;
}

// Merge the sorted batch b[0..nb) (no empty entries) into the sorted list t[0..L),
// writing the first L of the union to o (rank merge, merge_top gpu_graph.cu:162-222).
// With `recycle`, list entries pushed out that carry kInRange are appended in order to
// ev (merge_top_with_recycle_list, gpu_graph.cu:482-581); returns how many.
__device__ __forceinline__ uint32_t merge_list(const float* td, const uint32_t* tw, float* od, uint32_t* ow,
                                               uint32_t L, const float* bd, const uint32_t* bw, uint32_t nb,
                                               float* evd, uint32_t* evw, bool recycle) {
    const uint32_t lane = lane_id();
    for (uint32_t j = lane; j < nb; j += 32) {
        float dj = bd[j];
        uint32_t wj = bw[j];
        uint32_t pos = j + count_below(td, tw, L, mkkey(dj, wj));
        if (pos < L) {
            od[pos] = dj;
            ow[pos] = wj;
        }
    }
    uint32_t nev = 0;
    for (uint32_t i0 = 0; i0 < L; i0 += 32) {
        uint32_t i = i0 + lane;
        bool ev = false;
        float di = 0.0f;
        uint32_t wi = kEmpty;
        if (i < L) {
            di = td[i];
            wi = tw[i];
            uint32_t pos = i + count_below(bd, bw, nb, mkkey(di, wi));
            if (pos < L) {
                od[pos] = di;
                ow[pos] = wi;
            } else {
                ev = recycle && wi != kEmpty && (wi & kInRange);
            }
        }
        uint32_t m = __ballot_sync(kFull, ev);
        if (ev) {
            uint32_t k = nev + __popc(m & lanemask_lt());
            evd[k] = di;
            evw[k] = wi;
        }
        nev += __popc(m);
    }
    __syncwarp();
    return nev;
}

// Visited hash (open addressing, linear probing) keyed by position.
__device__ __forceinline__ uint32_t hash_slot(uint32_t key, uint32_t shift) { return (key * 2654435761u) >> shift; }

// Returns true when `key` was absent and is now inserted.  The table is kept at most
// half full, so a free slot always exists.
__device__ __forceinline__ bool hash_insert(uint32_t* H, uint32_t hs, uint32_t shift, uint32_t key) {
    uint32_t h = hash_slot(key, shift);
    for (uint32_t t = 0; t < hs; ++t) {
        uint32_t old = atomicCAS(&H[h], kEmpty, key);
        if (old == kEmpty) return true;
        if (old == key) return false;
        h = (h + 1) & (hs - 1);
    }
    return true;
}

__device__ __forceinline__ bool hash_contains(const uint32_t* H, uint32_t hs, uint32_t shift, uint32_t key) {
    uint32_t h = hash_slot(key, shift);
    for (uint32_t t = 0; t < hs; ++t) {
        uint32_t v = H[h];
        if (v == key) return true;
        if (v == kEmpty) return false;
        h = (h + 1) & (hs - 1);
    }
    return false;
}

__device__ __forceinline__ void hash_clear(uint32_t* H, uint32_t hs) {
    for (uint32_t i = lane_id(); i < hs; i += 32) H[i] = kEmpty;
    __syncwarp();
}

}  // namespace dev
}  // namespace gf
