// Query planning: which grid cells each query box overlaps, in cluster-guided order.
// Re-design of intersection_area_mark_little_seg_V2 (real_dataset_adapter.cuh:390-519:
// a marking kernel + copy_if/gather/reduce_by_key/exclusive_scan over a qnum x cells
// flag matrix + a qnum x N box-count pass) and get_partitions_access_order_V2
// (gpu_graph.cu:11742-11845: fp16 WMMA query x centroid distances written as a
// qnum x C matrix, a top-4 selection kernel, a per-query bitonic sort).
// Here: a count kernel + one scan + a fill kernel write the cell lists directly in
// increasing cell id; one tiled kernel computes query-centroid distances and keeps
// the 4 nearest in registers (the distance matrix never reaches HBM); one warp per
// query scores and sorts its cells.  The box-count pass runs only when --prefilter > 0
// (with prefilter 0 it can only select queries whose box is empty, whose result is
// empty on either route).
#include <cub/cub.cuh>

#include <algorithm>
#include <cstring>

#include "gf_device.cuh"
#include "gf_internal.h"

namespace gf {
namespace {

using namespace dev;

struct Slices {
    uint32_t lo[kMaxAttr], hi[kMaxAttr];
    bool empty;
};

// Slice range of each dimension (real_dataset_adapter.cuh:168-176):
// lo = first slice whose r_quant >= l, hi = last slice whose l_quant <= r.
__device__ __forceinline__ Slices slices_of(const float* lb, const float* rb, uint32_t a, const uint32_t* grid,
                                            const float* lq, const float* rq) {
    Slices s;
    s.empty = false;
    uint32_t off = 0;
    for (uint32_t j = 0; j < a; ++j) {
        uint32_t g = grid[j], k;
        for (k = 0; k < g && rq[off + k] < lb[j]; ++k) {
        }
        s.lo[j] = k;
        for (k = 0; k < g && lq[off + k] <= rb[j]; ++k) {
        }
        s.hi[j] = k - 1;
        if (k == 0 || s.lo[j] >= g || k - 1 < s.lo[j]) s.empty = true;
        off += g;
    }
    return s;
}

__global__ void plan_count_kernel(const float* __restrict__ lb, const float* __restrict__ rb, uint32_t qnum,
                                  uint32_t a, const uint32_t* __restrict__ grid, const float* __restrict__ lq,
                                  const float* __restrict__ rq, uint32_t* __restrict__ counts) {
    uint32_t q = blockIdx.x * blockDim.x + threadIdx.x;
    if (q >= qnum) return;
    Slices s = slices_of(lb + (size_t)q * a, rb + (size_t)q * a, a, grid, lq, rq);
    uint32_t c = 1;
    for (uint32_t j = 0; j < a; ++j) c *= s.empty ? 0 : (s.hi[j] - s.lo[j] + 1);
    counts[q] = s.empty ? 0 : c;
}

// Cells of each query in increasing cell id: cell = sum_j idx_j * prod_{k>j} grid_k
// (gpu_graph.cu:10965-10973), enumerated with the last dimension fastest.
__global__ void plan_fill_kernel(const float* __restrict__ lb, const float* __restrict__ rb, uint32_t qnum,
                                 uint32_t a, const uint32_t* __restrict__ grid, const float* __restrict__ lq,
                                 const float* __restrict__ rq, const uint32_t* __restrict__ counts,
                                 const uint32_t* __restrict__ offsets, uint32_t* __restrict__ cells) {
    uint32_t q = blockIdx.x * blockDim.x + threadIdx.x;
    if (q >= qnum || counts[q] == 0) return;
    Slices s = slices_of(lb + (size_t)q * a, rb + (size_t)q * a, a, grid, lq, rq);
    uint32_t idx[kMaxAttr];
    for (uint32_t j = 0; j < a; ++j) idx[j] = s.lo[j];
    uint32_t* out = cells + offsets[q];
    uint32_t n = 0;
    for (;;) {
        uint32_t pid = 0, f = 1;
        for (int j = (int)a - 1; j >= 0; --j) {
            pid += idx[j] * f;
            f *= grid[j];
        }
        out[n++] = pid;
        int j = (int)a - 1;
        while (j >= 0) {
            if (++idx[j] <= s.hi[j]) break;
            idx[j] = s.lo[j];
            --j;
        }
        if (j < 0) break;
    }
}

// Points inside each query box, over all n points (prefiltering_tag_elements,
// real_dataset_adapter.cuh:347-387).  Block: 256 threads x 8 queries; each thread
// tests its points against the 8 boxes held in shared memory.
constexpr uint32_t kBoxQ = 8;
__global__ void box_count_kernel(const float* __restrict__ attrs, uint32_t n, uint32_t a,
                                 const float* __restrict__ lb, const float* __restrict__ rb, uint32_t qnum,
                                 uint32_t* __restrict__ box) {
    __shared__ float sl[kBoxQ * kMaxAttr], sr[kBoxQ * kMaxAttr];
    __shared__ uint32_t red[kBoxQ];
    const uint32_t q0 = blockIdx.y * kBoxQ;
    for (uint32_t i = threadIdx.x; i < kBoxQ * a; i += blockDim.x) {
        uint32_t q = q0 + i / a;
        sl[i] = q < qnum ? lb[(size_t)q0 * a + i] : 1.0f;
        sr[i] = q < qnum ? rb[(size_t)q0 * a + i] : 0.0f;
    }
    if (threadIdx.x < kBoxQ) red[threadIdx.x] = 0;
    __syncthreads();
    uint32_t cnt[kBoxQ] = {0, 0, 0, 0, 0, 0, 0, 0};
    const uint32_t chunk = (n + gridDim.x - 1) / gridDim.x;
    const uint32_t beg = blockIdx.x * chunk, end = min(n, beg + chunk);
    for (uint32_t i = beg + threadIdx.x; i < end; i += blockDim.x) {
        float v[kMaxAttr];
        for (uint32_t j = 0; j < a; ++j) v[j] = __ldg(attrs + (size_t)i * a + j);
#pragma unroll
        for (uint32_t t = 0; t < kBoxQ; ++t) {
            bool ok = true;
            for (uint32_t j = 0; j < a; ++j) ok = ok && v[j] >= sl[t * a + j] && v[j] <= sr[t * a + j];
            cnt[t] += ok;
        }
    }
#pragma unroll
    for (uint32_t t = 0; t < kBoxQ; ++t) {
        uint32_t c = cnt[t];
        for (int o = 16; o > 0; o >>= 1) c += __shfl_down_sync(kFull, c, o);
        if ((threadIdx.x & 31) == 0 && c) atomicAdd(&red[t], c);
    }
    __syncthreads();
    if (threadIdx.x < kBoxQ && q0 + threadIdx.x < qnum && red[threadIdx.x])
        atomicAdd(&box[q0 + threadIdx.x], red[threadIdx.x]);
}

// Four nearest centroids per query (dis_cal_tensor_core + select_topk_by_reduce_min,
// tools.cuh:1399-1537), distances by one fma chain over d (oracle orc_dist_seq), ties
// by centroid id.  Block (x, y): 64 queries x the y-th range of c_chunk (<= 128)
// centroids; thread t owns queries 8*(t%8)..+7 and centroids 4*(t/8)..+3 and keeps their
// 32 distances in registers, each one sequential fma chain over the dimensions.  Query and
// centroid tiles of kTD dimensions are staged dimension-major in shared memory (float4
// global loads), so a step reads three float4 for 32 fused multiply-adds.  The finished
// 64 x 128 distance tile goes through shared memory, where 4 threads per query select its
// 4 best of the range (part (q, y)); a second kernel merges the ranges.
constexpr uint32_t kTQ = 64, kTC = 128, kTD = 32;
constexpr uint32_t kTileWords = kTD * (kTQ + kTC);
__global__ void __launch_bounds__(256) centroid_top4_kernel(const float* __restrict__ queries, uint32_t qnum,
                                                            uint32_t dim, const float* __restrict__ cent,
                                                            uint32_t C, uint32_t c_chunk, float* __restrict__ part_d,
                                                            uint32_t* __restrict__ part_i,
                                                            const uint32_t* __restrict__ live) {
    // staging tiles (qt: kTD x kTQ, ct: kTD x kTC), then the distance tile (kTQ x kTC)
    __shared__ __align__(16) float sm[kTQ * kTC > kTileWords ? kTQ * kTC : kTileWords];
    float* qt = sm;
    float* ct = sm + kTD * kTQ;
    const uint32_t t = threadIdx.x, qg = t & 7, cg = t >> 3;
    const uint32_t q0 = blockIdx.x * kTQ;
    const uint32_t qn = live ? min(live[0], qnum) : qnum;  // rows in use (a shard's listed queries)
    if (q0 >= qn) return;
    const uint32_t cbeg = blockIdx.y * c_chunk, cend = min(C, cbeg + c_chunk);
    f2x acc2[8][2];  // (query i, centroid pair j) partial distances, fp32 pairs
#pragma unroll
    for (int i = 0; i < 8; ++i) acc2[i][0] = acc2[i][1] = 0ull;
    const bool vec = (dim & 3u) == 0;
    for (uint32_t d0 = 0; d0 < dim; d0 += kTD) {
        __syncthreads();
        // rows x kTD/4 float4 groups; lanes take consecutive rows at the same dimensions,
        // so the transposed shared-memory stores hit different banks
        for (uint32_t e = t; e < (kTQ + kTC) * (kTD / 4); e += blockDim.x) {
            const bool isq = e < kTQ * (kTD / 4);
            const uint32_t e2 = isq ? e : e - kTQ * (kTD / 4);
            const uint32_t rows = isq ? kTQ : kTC;
            const uint32_t r = e2 % rows, dd = (e2 / rows) * 4;
            const uint32_t g = (isq ? q0 : cbeg) + r, lim = isq ? qn : cend;
            const float* src = isq ? queries : cent;
            float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            if (g < lim) {
                const uint32_t d = d0 + dd;
                if (vec && d + 3 < dim) {
                    const float4 x = *reinterpret_cast<const float4*>(src + (size_t)g * dim + d);
                    v[0] = x.x;
                    v[1] = x.y;
                    v[2] = x.z;
                    v[3] = x.w;
                } else {
#pragma unroll
                    for (uint32_t i = 0; i < 4; ++i)
                        if (d + i < dim) v[i] = src[(size_t)g * dim + d + i];
                }
            }
            float* dst = isq ? qt : ct;
#pragma unroll
            for (uint32_t i = 0; i < 4; ++i) dst[(dd + i) * rows + r] = v[i];
        }
        __syncthreads();
        const uint32_t dn = min(kTD, dim - d0);
        for (uint32_t dd = 0; dd < dn; ++dd) {
            const float4 qa4 = *reinterpret_cast<const float4*>(&qt[dd * kTQ + qg * 8]);
            const float4 qb4 = *reinterpret_cast<const float4*>(&qt[dd * kTQ + qg * 8 + 4]);
            const ulonglong2 cv = *reinterpret_cast<const ulonglong2*>(&ct[dd * kTC + cg * 4]);
            const float qa[8] = {qa4.x, qa4.y, qa4.z, qa4.w, qb4.x, qb4.y, qb4.z, qb4.w};
            // packed pairs of centroids (j, j+1): two independent IEEE operations each
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const f2x qq = pack2(qa[i], qa[i]);
                acc2[i][0] = sqacc2(sub2(qq, cv.x), acc2[i][0]);
                acc2[i][1] = sqacc2(sub2(qq, cv.y), acc2[i][1]);
            }
        }
    }
    __syncthreads();
    float* dt = sm;  // kTQ x kTC distances
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            dt[(qg * 8 + i) * kTC + cg * 4 + 2 * j] = lo2(acc2[i][j]);
            dt[(qg * 8 + i) * kTC + cg * 4 + 2 * j + 1] = hi2(acc2[i][j]);
        }
    __syncthreads();
    // 4 threads per query, 32 centroids each, then a 4-way merge over shuffles
    const uint32_t ql = t >> 2, part = t & 3;
    float bd[4];
    uint32_t bi[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) {  // all-ones key: above every distance, NaN (empty cluster) included
        bd[r] = __int_as_float(0xffffffff);
        bi[r] = kEmpty;
    }
    auto insert = [&](float dv, uint32_t c) {
        if (!(mkkey(dv, c) < mkkey(bd[3], bi[3]))) return;
        bd[3] = dv;
        bi[3] = c;
#pragma unroll
        for (int r = 3; r > 0; --r)
            if (mkkey(bd[r], bi[r]) < mkkey(bd[r - 1], bi[r - 1])) {
                const float td = bd[r];
                bd[r] = bd[r - 1];
                bd[r - 1] = td;
                const uint32_t ti = bi[r];
                bi[r] = bi[r - 1];
                bi[r - 1] = ti;
            }
    };
    for (uint32_t k = 0; k < kTC / 4; ++k) {
        const uint32_t cl = part * (kTC / 4) + ((k + ql) & (kTC / 4 - 1));  // rotation spreads banks
        const uint32_t c = cbeg + cl;
        if (c < cend) insert(dt[ql * kTC + cl], c);
    }
#pragma unroll
    for (int o = 1; o <= 2; o <<= 1) {
        float od[4];
        uint32_t oi[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            od[r] = __shfl_xor_sync(0xFFFFFFFFu, bd[r], o);
            oi[r] = __shfl_xor_sync(0xFFFFFFFFu, bi[r], o);
        }
#pragma unroll
        for (int r = 0; r < 4; ++r)
            if (oi[r] != kEmpty) insert(od[r], oi[r]);
    }
    if (part == 0 && q0 + ql < qn) {
        const size_t o = ((size_t)(q0 + ql) * gridDim.y + blockIdx.y) * 4;
        for (int r = 0; r < 4; ++r) {
            part_d[o + r] = bd[r];
            part_i[o + r] = bi[r];
        }
    }
}

// Merge the per-range candidates of each query into its 4 nearest centroids.  With a
// list `live` (shard planning), row q is query live[1 + q] and rows from live[0] on are unused.
__global__ void centroid_merge_kernel(uint32_t qnum, uint32_t splits, const float* __restrict__ part_d,
                                      const uint32_t* __restrict__ part_i, uint32_t* __restrict__ top4,
                                      const uint32_t* __restrict__ live) {
    const uint32_t q = blockIdx.x * blockDim.x + threadIdx.x;
    if (q >= (live ? min(live[0], qnum) : qnum)) return;
    float fd[4];
    uint32_t fi[4];
    for (int r = 0; r < 4; ++r) {
        fd[r] = __int_as_float(0xffffffff);
        fi[r] = kEmpty;
    }
    for (uint32_t e = 0; e < splits * 4; ++e) {
        const float dv = part_d[(size_t)q * splits * 4 + e];
        const uint32_t c = part_i[(size_t)q * splits * 4 + e];
        if (c == kEmpty || !(mkkey(dv, c) < mkkey(fd[3], fi[3]))) continue;
        fd[3] = dv;
        fi[3] = c;
        for (int k = 3; k > 0 && mkkey(fd[k], fi[k]) < mkkey(fd[k - 1], fi[k - 1]); --k) {
            float td = fd[k];
            fd[k] = fd[k - 1];
            fd[k - 1] = td;
            uint32_t ti = fi[k];
            fi[k] = fi[k - 1];
            fi[k - 1] = ti;
        }
    }
    const size_t out = live ? live[1 + q] : q;
    for (int r = 0; r < 4; ++r) top4[out * 4 + r] = fi[r];
}

// Score = sum over the 4 nearest centroids of hist[cell][centroid]; cells ordered by
// decreasing score, ties by increasing cell id (sort_by_clustering_info_weighted,
// gpu_graph.cu:11344-11396).  One warp per query; rank sort over the query's cells.  With
// a list `live` (shard planning) warp j orders query live[1 + j], for j < live[0].
constexpr uint32_t kMaxSortCells = 1024;
__global__ void order_cells_kernel(uint32_t qnum, const uint32_t* __restrict__ counts,
                                   const uint32_t* __restrict__ offsets, uint32_t* __restrict__ cells,
                                   const uint32_t* __restrict__ top4, const uint32_t* __restrict__ hist, uint32_t C,
                                   const uint32_t* __restrict__ live) {
    __shared__ uint64_t keys[4][kMaxSortCells];
    const uint32_t w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint32_t q = blockIdx.x * 4 + w;
    if (live) {
        if (q >= min(live[0], qnum)) return;
        q = live[1 + q];
    } else if (q >= qnum) {
        return;
    }
    const uint32_t m = counts[q];
    if (m <= 1) return;
    uint32_t* cl = cells + offsets[q];
    uint32_t t4[4];
    for (int r = 0; r < 4; ++r) t4[r] = top4[(size_t)q * 4 + r];
    for (uint32_t i = lane; i < m; i += 32) {
        uint32_t c = cl[i];
        uint32_t sc = 0;
        for (int r = 0; r < 4; ++r)
            if (t4[r] != kEmpty) sc += hist[(size_t)c * C + t4[r]];
        keys[w][i] = ((uint64_t)(0xFFFFFFFFu - sc) << 32) | c;
    }
    __syncwarp();
    for (uint32_t i = lane; i < m; i += 32) {
        uint64_t k = keys[w][i];
        uint32_t rank = 0;
        for (uint32_t j = 0; j < m; ++j) rank += keys[w][j] < k;
        cl[rank] = (uint32_t)k;
    }
}

// Shard planning: a shard searches only its own cells, so a query's cell order changes its
// results there only when two or more of its cells are the shard's.  Those queries are
// listed in live[1..] (live[0] = their number; list order is arbitrary, each query's
// planning is independent of its row) and their fp32 rows gathered into rows[j * dim].
// One warp per query.
__global__ void local_queries_kernel(uint32_t qnum, const uint32_t* __restrict__ counts,
                                     const uint32_t* __restrict__ offsets, const uint32_t* __restrict__ cells,
                                     const int32_t* __restrict__ slot, const float* __restrict__ q32, uint32_t dim,
                                     uint32_t* __restrict__ live, float* __restrict__ rows) {
    const uint32_t w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t q = blockIdx.x * 4 + w;
    if (q >= qnum) return;
    const uint32_t m = counts[q];
    const uint32_t* cl = cells + offsets[q];
    uint32_t held = 0;
    for (uint32_t i0 = 0; i0 < m && held < 2; i0 += 32) {
        const uint32_t i = i0 + lane;
        held += __popc(__ballot_sync(0xFFFFFFFFu, i < m && slot[cl[i]] >= 0));
    }
    if (held < 2) return;
    uint32_t j = 0;
    if (lane == 0) {
        j = atomicAdd(live, 1u);
        live[1 + j] = q;
    }
    j = __shfl_sync(0xFFFFFFFFu, j, 0);
    for (uint32_t k = lane; k < dim; k += 32) rows[(size_t)j * dim + k] = q32[(size_t)q * dim + k];
}

// Task order: queries with more cells first (gpu_graph.cu:12485-12493).
__global__ void iota_kernel(uint32_t* v, uint32_t n) {
    uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) v[i] = i;
}

}  // namespace

uint32_t centroid_chunk(uint32_t C) {
    uint32_t S = centroid_splits(C);
    uint32_t chunk = (C + S - 1) / std::max(S, 1u);
    return (chunk + kTC - 1) / kTC * kTC;
}

uint32_t centroid_splits(uint32_t C) {
    if (C == 0) return 1;  // no clusters: cells keep their id order
    uint32_t S = (C + kTC - 1) / kTC;
    S = std::min(S, 32u);
    S = std::max(S, 1u);
    // all ranges non-empty
    uint32_t chunk = ((C + S - 1) / S + kTC - 1) / kTC * kTC;
    return std::max(1u, (C + chunk - 1) / chunk);
}

gf_status plan_queries(gf_index* idx, gf_plan* plan, const float* queries, const float* lb, const float* rb,
                       uint32_t qnum, float prefilter, cudaStream_t s) {
    DeviceIndex& d = idx->d;
    Plan& p = plan->p;
    if (qnum > p.max_q) return fail(GF_ERR_ARG, "more queries than the plan was created for");
    if (qnum && (!queries || !lb || !rb)) return fail(GF_ERR_ARG, "null query arrays");
    p.planned = false;
    p.qnum = qnum;
    p.prefilter = prefilter;
    p.stream = s;
    if (qnum == 0) {
        p.planned = true;
        return GF_OK;
    }
    const uint32_t a = d.a;
    GF_CUDA(cudaMemcpyAsync(p.lb, lb, sizeof(float) * qnum * a, cudaMemcpyDeviceToDevice, s));
    GF_CUDA(cudaMemcpyAsync(p.rb, rb, sizeof(float) * qnum * a, cudaMemcpyDeviceToDevice, s));
    GF_CUDA(cudaMemcpyAsync(p.q32, queries, sizeof(float) * qnum * d.dim, cudaMemcpyDeviceToDevice, s));
    // planner counters, read by gf_search_stats_read: scratch[8] tensor-core waits that ran out,
    // [9] queries that fell back to the exact centroid scan, [10] centroids re-ranked exactly
    GF_CUDA(cudaMemsetAsync(p.scratch + 8, 0, 3 * sizeof(uint32_t), s));
    // 4 nearest centroids of rows[0 .. qnum) (with `live`: of the listed rows) into top4
    auto centroids = [&](cudaStream_t cs, const float* rows, const uint32_t* live) -> gf_status {
        if (p.S && centroid_tc_usable(d)) {  // tensor-core products + exact re-rank
            return centroid_top4_tc(d, rows, qnum, p.S, p.top4, p.scratch + 8, cs, live);
        }
        const uint32_t S = centroid_splits(d.C), chunk = centroid_chunk(d.C);
        dim3 grid((qnum + kTQ - 1) / kTQ, S);
        centroid_top4_kernel<<<grid, 256, 0, cs>>>(rows, qnum, d.dim, d.centroids, d.C, chunk, p.part_d, p.part_i,
                                                   live);
        centroid_merge_kernel<<<(qnum + 127) / 128, 128, 0, cs>>>(qnum, S, p.part_d, p.part_i, p.top4, live);
        GF_CUDA(cudaGetLastError());
        return GF_OK;
    };
    // On a whole index the centroid top-4 needs only the query rows: it runs on the plan's
    // side stream while this stream builds the cell lists and the task order, and the cell
    // order waits for both.  A shard lists its multi-cell queries from the cell lists first
    // (the grids stay sized for qnum; blocks past the device-side count return at once, so
    // the host never waits), so there everything stays on this stream.
    const bool fork = d.C && p.side && !p.live;
    if (fork) {
        GF_CUDA(cudaEventRecord(p.ev_fork, s));
        GF_CUDA(cudaStreamWaitEvent(p.side, p.ev_fork, 0));
        gf_status st = centroids(p.side, p.q32, nullptr);
        if (st != GF_OK) return st;
        GF_CUDA(cudaEventRecord(p.ev_join, p.side));
    }
    launch_f2h(p.q32, qnum, d.dim, d.d8, d.alpha, p.q16, s);
    const uint32_t tb = 128, nb = (qnum + tb - 1) / tb;
    plan_count_kernel<<<nb, tb, 0, s>>>(p.lb, p.rb, qnum, a, d.grid_d, d.lq_d, d.rq_d, p.counts);
    size_t tmp = p.scan_tmp_bytes;
    GF_CUDA(cub::DeviceScan::ExclusiveSum(p.scan_tmp, tmp, p.counts, p.offsets, (int)qnum, s));
    plan_fill_kernel<<<nb, tb, 0, s>>>(p.lb, p.rb, qnum, a, d.grid_d, d.lq_d, d.rq_d, p.counts, p.offsets,
                                       p.cells);
    const uint32_t* live = nullptr;
    if (d.C && !fork) {
        const float* rows = p.q32;
        if (p.live) {
            GF_CUDA(cudaMemsetAsync(p.live, 0, sizeof(uint32_t), s));
            GF_CUDA(cudaMemsetAsync(p.top4, 0xFF, sizeof(uint32_t) * 4 * qnum, s));
            local_queries_kernel<<<(qnum + 3) / 4, 128, 0, s>>>(qnum, p.counts, p.offsets, p.cells, d.sh_slot,
                                                                p.q32, d.dim, p.live, p.lq32);
            rows = p.lq32;
            live = p.live;
        }
        gf_status st = centroids(s, rows, live);
        if (st != GF_OK) return st;
    }
    if (prefilter > 0.0f) {
        if (d.at_ok) {
            box_count_tiles(d, p.lb, p.rb, qnum, p.box, s);
        } else {
            GF_CUDA(cudaMemsetAsync(p.box, 0, sizeof(uint32_t) * qnum, s));
            dim3 grid(std::min<uint32_t>((d.n + 256 * 64 - 1) / (256 * 64), 1024), (qnum + kBoxQ - 1) / kBoxQ);
            box_count_kernel<<<grid, 256, 0, s>>>(d.attrs, d.n, a, p.lb, p.rb, qnum, p.box);
        }
    }
    // processing order: most cells first
    iota_kernel<<<nb, tb, 0, s>>>(p.task + p.max_q, qnum);
    size_t tmp2 = p.scan_tmp_bytes;
    GF_CUDA(cub::DeviceRadixSort::SortPairsDescending(p.scan_tmp, tmp2, p.counts, p.task + 2 * p.max_q,
                                                      p.task + p.max_q, p.task, (int)qnum, 0,
                                                      count_sort_bits(d.ncells), s));
    if (d.C) {
        if (fork) GF_CUDA(cudaStreamWaitEvent(s, p.ev_join, 0));
        order_cells_kernel<<<(qnum + 3) / 4, 128, 0, s>>>(qnum, p.counts, p.offsets, p.cells, p.top4, d.hist, d.C,
                                                          live);
    } else {
        GF_CUDA(cudaMemsetAsync(p.top4, 0xFF, sizeof(uint32_t) * 4 * qnum, s));
    }
    GF_CUDA(cudaGetLastError());
    p.planned = true;
    return GF_OK;
}

}  // namespace gf

using namespace gf;

namespace {
struct DeviceGuard2 {
    int prev = -1;
    explicit DeviceGuard2(int d) {
        cudaGetDevice(&prev);
        cudaSetDevice(d);
    }
    ~DeviceGuard2() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

void free_plan(Plan& p) {
    void* ptrs[] = {p.S, p.q16, p.q32, p.lb, p.rb, p.counts, p.offsets, p.cells, p.top4, p.box, p.task, p.scratch,
                    p.stats, p.scan_tmp, p.part_d, p.part_i, p.live, p.lq32};
    for (void* x : ptrs)
        if (x) cudaFree(x);
    if (p.io) cudaFree(p.io);
    if (p.xmark) cudaFree(p.xmark);
    if (p.ev_fork) cudaEventDestroy(p.ev_fork);
    if (p.ev_join) cudaEventDestroy(p.ev_join);
    if (p.side) cudaStreamDestroy(p.side);
    if (p.flags_h) cudaFreeHost(p.flags_h);
    p.flags_h = nullptr;
    p.side = nullptr;
    p.ev_fork = p.ev_join = nullptr;
    if (p.run) cudaFree(p.run);
    free_batch_state(p.batch);
    p.batch = nullptr;
}
}  // namespace

extern "C" {

gf_status gf_plan_create(gf_index* idx, uint32_t max_queries, gf_plan** out) {
    if (!idx || !out) return fail(GF_ERR_ARG, "null argument");
    if (max_queries == 0) return fail(GF_ERR_ARG, "max_queries must be > 0");
    *out = nullptr;
    DeviceIndex& d = idx->d;
    DeviceGuard2 guard(d.device);
    gf_plan* pl = new gf_plan();
    Plan& p = pl->p;
    p.idx = idx;
    p.device = d.device;
    p.max_q = max_queries;
    const size_t Q = max_queries;
    cudaError_t e = cudaSuccess;
    auto A = [&](void** ptr, size_t bytes) {
        if (e == cudaSuccess) e = cudaMalloc(ptr, std::max<size_t>(bytes, 16));
    };
    A((void**)&p.q16, Q * d.d8 * 2);
    A((void**)&p.q32, Q * d.dim * 4);
    A((void**)&p.lb, Q * d.a * 4);
    A((void**)&p.rb, Q * d.a * 4);
    A((void**)&p.counts, Q * 4);
    A((void**)&p.offsets, Q * 4);
    A((void**)&p.cells, Q * d.ncells * 4);
    A((void**)&p.top4, Q * 16);
    if (centroid_tc_usable(d)) A((void**)&p.S, Q * centroid_tc_stride(d) * 4);
    A((void**)&p.part_d, Q * centroid_splits(d.C) * 16);
    A((void**)&p.part_i, Q * centroid_splits(d.C) * 16);
    A((void**)&p.box, Q * 4);
    A((void**)&p.task, Q * 3 * 4);
    A((void**)&p.scratch, 64);
    if (e == cudaSuccess) e = cudaMallocHost((void**)&p.flags_h, 2 * sizeof(unsigned long long));
    if (d.sharded) {
        A((void**)&p.live, (Q + 1) * 4);
        A((void**)&p.lq32, Q * d.dim * 4);
    } else if (e == cudaSuccess && d.C) {
        e = cudaStreamCreateWithFlags(&p.side, cudaStreamNonBlocking);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p.ev_fork, cudaEventDisableTiming);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p.ev_join, cudaEventDisableTiming);
    }
    A((void**)&p.stats, 8 * sizeof(unsigned long long));
    if (e == cudaSuccess) {
        size_t t1 = 0, t2 = 0;
        cub::DeviceScan::ExclusiveSum(nullptr, t1, p.counts, p.offsets, (int)Q);
        cub::DeviceRadixSort::SortPairsDescending(nullptr, t2, p.counts, p.task, p.task, p.task, (int)Q, 0,
                                              count_sort_bits(d.ncells));
        p.scan_tmp_bytes = std::max(t1, t2);
        A(&p.scan_tmp, p.scan_tmp_bytes);
    }
    if (e != cudaSuccess) {
        gf_status st = cuda_fail(e, "plan buffers");
        free_plan(p);
        delete pl;
        return st;
    }
    if (d.ncells > kMaxSortCells) {
        free_plan(p);
        delete pl;
        return fail(GF_ERR_ARG, "more than 1024 cells per index are not supported by the planner");
    }
    *out = pl;
    return GF_OK;
}

gf_status gf_plan_destroy(gf_plan* plan) {
    if (!plan) return GF_OK;
    DeviceGuard2 guard(plan->p.device);
    free_plan(plan->p);
    delete plan;
    return GF_OK;
}

gf_status gf_plan_queries(gf_index* idx, gf_plan* plan, const float* queries, const float* lb, const float* rb,
                          uint32_t qnum, float prefilter, void* stream) {
    if (!idx || !plan || plan->p.idx != idx) return fail(GF_ERR_ARG, "plan does not belong to this index");
    DeviceGuard2 guard(idx->d.device);
    return plan_queries(idx, plan, queries, lb, rb, qnum, prefilter, (cudaStream_t)stream);
}

gf_status gf_plan_read(gf_plan* plan, uint32_t* counts, uint32_t* offsets, uint32_t* cells, uint64_t cap,
                       uint32_t* top4, uint32_t* box_counts) {
    if (!plan) return fail(GF_ERR_ARG, "null plan");
    Plan& p = plan->p;
    if (!p.planned) return fail(GF_ERR_STATE, "plan not built");
    DeviceGuard2 guard(p.device);
    GF_CUDA(cudaStreamSynchronize(p.stream));
    const uint32_t q = p.qnum;
    if (q == 0) return GF_OK;
    std::vector<uint32_t> c(q), o(q);
    GF_CUDA(cudaMemcpy(c.data(), p.counts, 4ull * q, cudaMemcpyDeviceToHost));
    GF_CUDA(cudaMemcpy(o.data(), p.offsets, 4ull * q, cudaMemcpyDeviceToHost));
    uint64_t total = (uint64_t)o[q - 1] + c[q - 1];
    if (counts) std::memcpy(counts, c.data(), 4ull * q);
    if (offsets) std::memcpy(offsets, o.data(), 4ull * q);
    if (cells) {
        if (total > cap) return fail(GF_ERR_ARG, "cells buffer too small");
        GF_CUDA(cudaMemcpy(cells, p.cells, 4ull * total, cudaMemcpyDeviceToHost));
    }
    if (top4) GF_CUDA(cudaMemcpy(top4, p.top4, 16ull * q, cudaMemcpyDeviceToHost));
    if (box_counts) GF_CUDA(cudaMemcpy(box_counts, p.box, 4ull * q, cudaMemcpyDeviceToHost));
    return GF_OK;
}

gf_status gf_search(gf_index* idx, gf_plan* plan, const gf_search_params* params, uint32_t* ids_out,
                    float* dist_out, void* stream) {
    if (!idx || !plan || plan->p.idx != idx) return fail(GF_ERR_ARG, "plan does not belong to this index");
    DeviceGuard2 guard(idx->d.device);
    return gf::search(idx, plan, params, ids_out, dist_out, (cudaStream_t)stream);
}

gf_status gf_search_stats_read(gf_plan* plan, gf_search_stats* out) {
    if (!plan || !out) return fail(GF_ERR_ARG, "null argument");
    Plan& p = plan->p;
    DeviceGuard2 guard(p.device);
    unsigned long long v[8];
    GF_CUDA(cudaStreamSynchronize(p.stream));
    GF_CUDA(cudaMemcpy(v, p.stats, sizeof(v), cudaMemcpyDeviceToHost));
    out->n_dist = v[0];
    out->n_exp = v[1];
    out->n_cross = v[2];
    out->n_hops = v[3];
    out->n_exact = v[4];
    out->n_queries = v[5];
    uint32_t pc[3];
    GF_CUDA(cudaMemcpy(pc, p.scratch + 8, sizeof(pc), cudaMemcpyDeviceToHost));
    out->n_timeouts = v[7] + pc[0];
    out->n_plan_fallbacks = pc[1];
    out->n_plan_reranked = pc[2];
    return GF_OK;
}

gf_status gf_search_host(gf_index* idx, gf_plan* plan, const gf_search_params* params, const float* queries_host,
                         const float* lb_host, const float* rb_host, uint32_t qnum, float prefilter,
                         uint32_t* ids_host, float* dist_host, void* stream) {
    if (!idx || !plan || plan->p.idx != idx) return fail(GF_ERR_ARG, "plan does not belong to this index");
    if (qnum > plan->p.max_q) return fail(GF_ERR_ARG, "more queries than the plan was created for");
    if (qnum && (!queries_host || !lb_host || !rb_host || !ids_host)) return fail(GF_ERR_ARG, "null host array");
    DeviceGuard2 guard(idx->d.device);
    DeviceIndex& d = idx->d;
    Plan& p = plan->p;
    cudaStream_t s = (cudaStream_t)stream;
    gf_search_params P;
    gf_search_defaults(&P);
    if (params) P = *params;
    // device copies of the host arrays, in one buffer owned by the plan
    const size_t need = std::max<size_t>((size_t)qnum * (d.dim + 2 * d.a + 2 * P.k), 1) * 4;
    cudaError_t e = cudaSuccess;
    if (need > p.io_bytes) {
        if (p.io) {
            if ((e = cudaStreamSynchronize(s)) != cudaSuccess) return cuda_fail(e, "gf_search_host");
            cudaFree(p.io);
            p.io = nullptr;
            p.io_bytes = 0;
        }
        if ((e = cudaMalloc(&p.io, need)) != cudaSuccess) return cuda_fail(e, "gf_search_host staging buffer");
        p.io_bytes = need;
    }
    float* dq = static_cast<float*>(p.io);
    float* dl = dq + (size_t)qnum * d.dim;
    float* dr = dl + (size_t)qnum * d.a;
    uint32_t* dids = reinterpret_cast<uint32_t*>(dr + (size_t)qnum * d.a);
    float* ddist = reinterpret_cast<float*>(dids + (size_t)qnum * P.k);
    gf_status st = GF_OK;
    do {
        if ((e = cudaMemcpyAsync(dq, queries_host, 4ull * qnum * d.dim, cudaMemcpyHostToDevice, s)) != cudaSuccess) break;
        if ((e = cudaMemcpyAsync(dl, lb_host, 4ull * qnum * d.a, cudaMemcpyHostToDevice, s)) != cudaSuccess) break;
        if ((e = cudaMemcpyAsync(dr, rb_host, 4ull * qnum * d.a, cudaMemcpyHostToDevice, s)) != cudaSuccess) break;
        st = plan_queries(idx, plan, dq, dl, dr, qnum, prefilter, s);
        if (st != GF_OK) break;
        st = gf::search(idx, plan, &P, dids, dist_host ? ddist : nullptr, s);
        if (st != GF_OK) break;
        if ((e = cudaMemcpyAsync(ids_host, dids, 4ull * qnum * P.k, cudaMemcpyDeviceToHost, s)) != cudaSuccess) break;
        if (dist_host &&
            (e = cudaMemcpyAsync(dist_host, ddist, 4ull * qnum * P.k, cudaMemcpyDeviceToHost, s)) != cudaSuccess)
            break;
        // the search's and the planner's timeout counters come back with the results
        p.flags_h[1] = 0;
        if ((e = cudaMemcpyAsync(p.flags_h, p.stats + 7, 8, cudaMemcpyDeviceToHost, s)) != cudaSuccess) break;
        if ((e = cudaMemcpyAsync(p.flags_h + 1, p.scratch + 8, 4, cudaMemcpyDeviceToHost, s)) != cudaSuccess) break;
        e = cudaStreamSynchronize(s);
        if (e == cudaSuccess && (p.flags_h[0] || p.flags_h[1])) st = fail(GF_ERR_TIMEOUT, "a bounded device wait ran out");
    } while (0);
    if (st != GF_OK) return st;
    if (e != cudaSuccess) return cuda_fail(e, "gf_search_host");
    return GF_OK;
}

gf_status gf_bruteforce(gf_index* idx, const float* queries, const float* lb, const float* rb, uint32_t qnum,
                        uint32_t k, uint32_t* ids_out, float* dist_out, void* stream) {
    if (!idx) return fail(GF_ERR_ARG, "null index");
    DeviceGuard2 guard(idx->d.device);
    return gf::bruteforce(idx, queries, lb, rb, qnum, k, ids_out, dist_out, (cudaStream_t)stream);
}

gf_status gf_bruteforce_ex(gf_index* idx, const float* queries, const float* lb, const float* rb, uint32_t qnum,
                           uint32_t k, uint32_t* ids_out, float* dist_out, const gf_bf_params* params, void* stream) {
    if (!idx) return fail(GF_ERR_ARG, "null index");
    DeviceGuard2 guard(idx->d.device);
    return gf::bruteforce(idx, queries, lb, rb, qnum, k, ids_out, dist_out, (cudaStream_t)stream, params);
}

}  // extern "C"
