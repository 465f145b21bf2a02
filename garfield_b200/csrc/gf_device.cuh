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

// 16-byte read-only load of a stored row chunk.
__device__ __forceinline__ uint4 ldg16(const uint4* p) { return __ldg(p); }

// Packed two-wide fp32 arithmetic (sm_100a): each half is an independent IEEE
// round-to-nearest operation, so the results equal the scalar ones bit for bit.
typedef unsigned long long f2x;  // (first, second) float in (low, high) 32 bits
__device__ __forceinline__ f2x pack2(float a, float b) {
    return ((f2x)__float_as_uint(b) << 32) | __float_as_uint(a);
}
__device__ __forceinline__ float lo2(f2x v) { return __uint_as_float((uint32_t)v); }
__device__ __forceinline__ float hi2(f2x v) { return __uint_as_float((uint32_t)(v >> 32)); }
__device__ __forceinline__ f2x sub2(f2x a, f2x b) {
    f2x d;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ f2x sqacc2(f2x d, f2x acc) {  // d*d + acc, fused, per half
    f2x r;
    asm("fma.rn.f32x2 %0, %1, %1, %2;" : "=l"(r) : "l"(d), "l"(acc));
    return r;
}
__device__ __forceinline__ f2x h2_to_f2x(uint32_t h) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h));
    return pack2(f.x, f.y);
}

__device__ __forceinline__ f2x mul2(f2x a, f2x b) {
    f2x r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ f2x fma2(f2x a, f2x b, f2x c) {  // a * b + c, fused, per half
    f2x r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
__device__ __forceinline__ f2x add2(f2x a, f2x b) {
    f2x r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}

// End of the canonical sum over the eight partials p[0..7], held as the packed pairs
// acc[j] = (p[2j], p[2j+1]): s[j] = p[j] + p[j+4], t[j] = s[j] + s[j+2], t[0] + t[1].
__device__ __forceinline__ float finish8(f2x a0, f2x a1, f2x a2, f2x a3) {
    const f2x t = add2(add2(a0, a2), add2(a1, a3));
    return __fadd_rn(lo2(t), hi2(t));
}

// Partial sums of one half of a staged row (oracle orc_dist16 / orc_dist8): the chunks
// of parity `half` (16-byte chunks: 8 fp16 or 16 byte elements), element i feeding packed
// partial pair (i mod 8) / 2.  Two lanes evaluate a row, one per half; the owner of half 0
// adds the other half's partials (add2) and finishes the sum (finish8).  The chunk loop
// stays rolled, which keeps the search kernel's instruction footprint small.

// (x - q) of an fp16 pair against an fp32 pair: one mixed-precision subtract per element
// (the fp16 operand is widened exactly and the difference rounded once, as a widening
// followed by an fp32 subtract would); (x - q)^2 == (q - x)^2, rounding being symmetric.
__device__ __forceinline__ f2x hsub_f2x(uint32_t h, f2x q) {
    float lo, hi;
    asm("{\n .reg .b16 a, b;\n mov.b32 {a, b}, %2;\n sub.rn.f32.f16 %0, a, %3;\n sub.rn.f32.f16 %1, b, %4;\n}\n"
        : "=f"(lo), "=f"(hi)
        : "r"(h), "f"(lo2(q)), "f"(hi2(q)));
    return pack2(lo, hi);
}

// fp16 rows: the query is held as fp32 pairs q2[c*4 .. c*4+3] of chunk c.
template <int NCH>
__device__ __forceinline__ void half16(const uint4* srow, const f2x* q2, uint32_t nch_rt, uint32_t half, f2x* p) {
    const uint32_t nch = NCH ? (uint32_t)NCH : nch_rt;
#pragma unroll 2
    for (uint32_t c = half; c < nch; c += 2) {
        const uint4 x = srow[c];
        const ulonglong2 qa = *reinterpret_cast<const ulonglong2*>(q2 + c * 4);
        const ulonglong2 qb = *reinterpret_cast<const ulonglong2*>(q2 + c * 4 + 2);
        p[0] = sqacc2(hsub_f2x(x.x, qa.x), p[0]);
        p[1] = sqacc2(hsub_f2x(x.y, qa.y), p[1]);
        p[2] = sqacc2(hsub_f2x(x.z, qb.x), p[2]);
        p[3] = sqacc2(hsub_f2x(x.w, qb.y), p[3]);
    }
}

// Byte element e (0..3) of w as the float 2^23 + byte (exact): the byte is placed under
// the exponent bits of 2^23 with one byte permute.
__device__ __forceinline__ float byte_f23(uint32_t w, uint32_t e) {
    return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7440u | e));
}

// Byte rows: element i contributes diff = fma(-scale[i], byte ^ xmask - bias[i], q[i]), the
// integer difference computed exactly as (2^23 + byte) - (2^23 + bias).  The decoded value
// is not rounded on its own: ptxas contracts a packed multiply followed by a packed subtract
// into one fused operation even when both carry .rn, so the fused form is the defined one
// and is written as such.  q2, ns2, b2: the query, -scale and 2^23 + bias as fp32 pairs.
template <int NCH>
__device__ __forceinline__ void half8(const uint4* srow, const f2x* q2, const f2x* ns2, const f2x* b2, uint32_t xmask,
                                      uint32_t nch_rt, uint32_t half, f2x* p) {
    const uint32_t nch = NCH ? (uint32_t)NCH : nch_rt;
#pragma unroll 2
    for (uint32_t c = half; c < nch; c += 2) {
        const uint4 x = srow[c];
        const uint32_t w[4] = {x.x ^ xmask, x.y ^ xmask, x.z ^ xmask, x.w ^ xmask};
#pragma unroll
        for (int j = 0; j < 8; ++j) {  // element pairs 2j, 2j+1 of the chunk -> partial pair j % 4
            const uint32_t word = w[j >> 1], e = (j & 1) * 2;
            const f2x u = pack2(byte_f23(word, e), byte_f23(word, e + 1));
            const uint32_t k = c * 8 + j;  // pair index in the row
            p[j & 3] = sqacc2(fma2(sub2(u, b2[k]), ns2[k], q2[k]), p[j & 3]);
        }
    }
}

// Canonical fp32 squared distance (oracle orc_dist32) of a global row of nch float4
// chunks against a query row in shared memory: chunk c covers elements 4c..4c+3, which
// feed the partial pairs 2(c mod 2) and 2(c mod 2)+1.  Eight chunks are loaded before
// they are accumulated, to keep several loads in flight.
__device__ __forceinline__ float dist32(const float4* __restrict__ row, const float4* __restrict__ q, uint32_t nch) {
    f2x p[4] = {0ull, 0ull, 0ull, 0ull};
    for (uint32_t c0 = 0; c0 < nch; c0 += 8) {
        float4 x[8];
#pragma unroll
        for (int u = 0; u < 8; ++u)
            if (c0 + u < nch) x[u] = __ldg(row + c0 + u);
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            if (c0 + u < nch) {
                const float4 qv = q[c0 + u];
                const int j = (u & 1) * 2;
                p[j] = sqacc2(sub2(pack2(qv.x, qv.y), pack2(x[u].x, x[u].y)), p[j]);
                p[j + 1] = sqacc2(sub2(pack2(qv.z, qv.w), pack2(x[u].z, x[u].w)), p[j + 1]);
            }
        }
    }
    return finish8(p[0], p[1], p[2], p[3]);
}

// Bulk (TMA) copies into shared memory, completed on a shared-memory mbarrier.
__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
// Order earlier generic-proxy accesses of shared memory before later bulk-copy writes.
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
// Copy `bytes` (multiple of 16, both addresses 16-byte aligned) from global to shared
// memory; completion is counted on `bar`.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
// Waits up to an implementation-defined time (suspend_ns is a hint) for the phase of
// parity `parity` to complete; false when it has not completed yet.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity, uint32_t suspend_ns) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(suspend_ns)
        : "memory");
    return ok != 0;
}

// 16-byte asynchronous global -> shared copy (cp.async, L2 only) and its fences.
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
    uint32_t d = (uint32_t)__cvta_generic_to_shared(smem_dst);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(d), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;\n" ::: "memory");
}

// Closed-box test of one point (merge_top_with_recycle_list's filter, gpu_graph.cu:514-520).
__device__ __forceinline__ bool in_box(const float* __restrict__ attrs, long long row, uint32_t a,
                                       const float* __restrict__ lb, const float* __restrict__ rb) {
    bool ok = true;  // no short-circuit: the attribute loads are independent
    for (uint32_t j = 0; j < a; ++j) {
        const float v = __ldg(attrs + row * a + j);
        ok &= (v >= lb[j]) & (v <= rb[j]);
    }
    return ok;
}

// Warp bitonic sort of (d, w) pairs in shared memory by mkkey; n is a power of two.
__device__ __forceinline__ void warp_sort(float* d, uint32_t* w, uint32_t n) {
    const uint32_t lane = lane_id();
    for (uint32_t lk = 1; (1u << lk) <= n; ++lk) {
        const uint32_t k = 1u << lk;
        for (int lj = (int)lk - 1; lj >= 0; --lj) {
            const uint32_t j = 1u << lj;
            for (uint32_t i = lane; i < (n >> 1); i += 32) {
                const uint32_t lo = ((i >> lj) << (lj + 1)) | (i & (j - 1));
                const uint32_t hi = lo + j;
                const bool asc = (lo & k) == 0;
                const float dl = d[lo], dh = d[hi];
                const uint32_t wl = w[lo], wh = w[hi];
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

// Bitonic sort of 32 (d, w) pairs held one per lane, ascending by mkkey, in registers.
__device__ __forceinline__ void warp_sort32(float& d, uint32_t& w) {
    const uint32_t lane = lane_id();
#pragma unroll
    for (uint32_t k = 2; k <= 32; k <<= 1) {
#pragma unroll
        for (uint32_t j = k >> 1; j > 0; j >>= 1) {
            const float od = __shfl_xor_sync(kFull, d, j);
            const uint32_t ow = __shfl_xor_sync(kFull, w, j);
            const uint64_t mk = mkkey(d, w), ok = mkkey(od, ow);
            const bool keep_min = ((lane & j) == 0) == ((lane & k) == 0);
            if (keep_min ? (ok < mk) : (ok > mk)) {
                d = od;
                w = ow;
            }
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

// H is 16-byte aligned and hs a multiple of 4 (a power of two >= 256)
__device__ __forceinline__ void hash_clear(uint32_t* H, uint32_t hs) {
    uint4* H4 = reinterpret_cast<uint4*>(H);
    for (uint32_t i = lane_id(); i < (hs >> 2); i += 32) H4[i] = make_uint4(kEmpty, kEmpty, kEmpty, kEmpty);
    __syncwarp();
}

}  // namespace dev
}  // namespace gf

namespace gf {
namespace dev {

// ------------------------------------------------------------------ 64-bit list keys
// A list entry is one 64-bit word that is also its sort key:
//   bits 63..32  distance (fp32 bits; distances are >= +0 so the bits order like values)
//   bits 31..2   cell-major position
//   bit 1        explored,  bit 0  in range
// Ordering by the word orders by (distance, position); the flag bits never decide an
// order because two entries never share a position.  kEmptyKey (all ones) sorts last.
typedef unsigned long long key_t;
constexpr key_t kEmptyKey = ~0ull;
constexpr uint32_t kKeyExplored = 2u, kKeyInRange = 1u;

__device__ __forceinline__ key_t make_key(float d, uint32_t pos, uint32_t flags) {
    return ((key_t)__float_as_uint(d) << 32) | ((key_t)pos << 2) | flags;
}
__device__ __forceinline__ uint32_t key_pos(key_t k) { return ((uint32_t)k) >> 2; }
__device__ __forceinline__ float key_dist(key_t k) { return __uint_as_float((uint32_t)(k >> 32)); }

__device__ __forceinline__ key_t shfl_xor_key(key_t k, uint32_t m) {
    uint32_t lo = __shfl_xor_sync(kFull, (uint32_t)k, m);
    uint32_t hi = __shfl_xor_sync(kFull, (uint32_t)(k >> 32), m);
    return ((key_t)hi << 32) | lo;
}

// Bitonic sort of 32 keys held one per lane, ascending.
__device__ __forceinline__ key_t warp_sort32_key(key_t k) {
    const uint32_t lane = lane_id();
#pragma unroll
    for (uint32_t s = 2; s <= 32; s <<= 1) {
#pragma unroll
        for (uint32_t j = s >> 1; j > 0; j >>= 1) {
            const key_t o = shfl_xor_key(k, j);
            const bool keep_min = ((lane & j) == 0) == ((lane & s) == 0);
            k = keep_min ? (o < k ? o : k) : (o > k ? o : k);
        }
    }
    return k;
}

// The same network stopped after the runs of `width` lanes (a power of two, warp-uniform):
// when every lane from `width` on holds kEmptyKey, lanes [0, width) end sorted ascending and
// the result equals the full sort (later lanes only ever meet lanes of their own run).
__device__ __forceinline__ key_t warp_sort_key_upto(key_t k, uint32_t width) {
    const uint32_t lane = lane_id();
#pragma unroll
    for (uint32_t s = 2; s <= 32; s <<= 1) {
        if (s > width) break;
#pragma unroll
        for (uint32_t j = s >> 1; j > 0; j >>= 1) {
            const key_t o = shfl_xor_key(k, j);
            const bool keep_min = ((lane & j) == 0) == ((lane & s) == 0);
            k = keep_min ? (o < k ? o : k) : (o > k ? o : k);
        }
    }
    return k;
}

// Bitonic sort of n (power of two) keys in shared memory, ascending.
__device__ __forceinline__ void warp_sort_keys(key_t* a, uint32_t n) {
    const uint32_t lane = lane_id();
    for (uint32_t ls = 1; (1u << ls) <= n; ++ls) {
        const uint32_t s = 1u << ls;
        for (int lj = (int)ls - 1; lj >= 0; --lj) {
            const uint32_t j = 1u << lj;
            for (uint32_t i = lane; i < (n >> 1); i += 32) {
                const uint32_t lo = ((i >> lj) << (lj + 1)) | (i & (j - 1));
                const uint32_t hi = lo + j;
                const key_t x = a[lo], y = a[hi];
                if ((x > y) == ((lo & s) == 0)) {
                    a[lo] = y;
                    a[hi] = x;
                }
            }
            __syncwarp();
        }
    }
}

// Number of keys of the sorted array a[0..n) below `key`.
__device__ __forceinline__ uint32_t keys_below(const key_t* a, uint32_t n, key_t key) {
    uint32_t lo = 0, hi = n;
    while (lo < hi) {
        const uint32_t mid = (lo + hi) >> 1;
        if (a[mid] < key)
            lo = mid + 1;
        else
            hi = mid;
    }
    return lo;
}

// Merge the sorted batch b[0..nb) (no empty keys) into the sorted list t[0..L), writing
// the first L keys of the union to o (t and o distinct).  Only the batch prefix that
// enters is processed, and list entries before the first insertion point are copied.
// With `recycle`, list entries pushed out that are in range are appended in order to ev
// (merge_top_with_recycle_list, gpu_graph.cu:482-581).  Returns (entered << 16) | evicted;
// entered == 0 means o was not written.
static __device__ __noinline__ uint32_t merge_keys(const key_t* t, key_t* o, uint32_t L, const key_t* b, uint32_t nb,
                                            key_t* ev, bool recycle) {
    const uint32_t lane = lane_id();
    // entering batch prefix: b[j] enters iff j + #(t < b[j]) < L (increasing in j)
    // (first: list entries before b[0]'s insertion point, lane 0's rank in the first pass)
    uint32_t m = 0, first = 0;
    for (uint32_t j0 = 0; j0 < nb; j0 += 32) {
        const uint32_t j = j0 + lane;
        uint32_t pos = 0xFFFFFFFFu;
        key_t kj = kEmptyKey;
        if (j < nb) {
            kj = b[j];
            pos = j + keys_below(t, L, kj);
        }
        if (j0 == 0) first = __shfl_sync(kFull, pos, 0);
        const uint32_t msk = __ballot_sync(kFull, pos < L);
        if (pos < L) o[pos] = kj;
        m += __popc(msk);
        if (__popc(msk) < 32) break;
    }
    if (m == 0) return 0;
    uint32_t nev = 0;
    for (uint32_t i0 = 0; i0 < L; i0 += 32) {
        const uint32_t i = i0 + lane;
        bool out = false;
        key_t ki = kEmptyKey;
        if (i < L) {
            ki = t[i];
            const uint32_t pos = i < first ? i : i + keys_below(b, m, ki);
            if (pos < L)
                o[pos] = ki;
            else
                out = recycle && ki != kEmptyKey && (ki & kKeyInRange);
        }
        const uint32_t msk = __ballot_sync(kFull, out);
        if (out) ev[nev + __popc(msk & lanemask_lt())] = ki;
        nev += __popc(msk);
    }
    __syncwarp();
    return (m << 16) | nev;
}

}  // namespace dev
}  // namespace gf
