// Index construction: host arrays in the reference's layout -> device-resident index in
// cell-major order.  Replaces the loading block of real_dataset_test_multiD
// (realdataset_search.cu:2118-2393): get_graph_info (check.cu:406-484), get_idx_mapper
// (tools.cuh:862-915), load_result of the global graph (tools.cuh:205-223), f2h
// (tools.cuh:308-321), load_clustering (tools.cuh:569-602).
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <random>
#include <string>

#include "gf_internal.h"

namespace gf {

static thread_local std::string g_err;

void set_error(const std::string& msg) { g_err = msg; }

gf_status fail(gf_status s, const std::string& msg) {
    g_err = msg;
    return s;
}

gf_status cuda_fail(cudaError_t e, const char* what) {
    g_err = std::string(what) + ": " + cudaGetErrorString(e);
    return e == cudaErrorMemoryAllocation ? GF_ERR_OOM : GF_ERR_CUDA;
}

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int d) {
        cudaGetDevice(&prev);
        cudaSetDevice(d);
    }
    ~DeviceGuard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

// half(x * alpha) per element, rows padded with zeros to d8 (tools.cuh:308-321).
__global__ void f2h_kernel(const float* __restrict__ in, uint32_t n, uint32_t dim, uint32_t d8, float alpha,
                           __half* __restrict__ out) {
    size_t total = (size_t)n * d8;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        size_t row = i / d8;
        uint32_t d = (uint32_t)(i - row * d8);
        float v = d < dim ? __fmul_rn(in[row * dim + d], alpha) : 0.0f;
        out[i] = __float2half_rn(v);
    }
}

void launch_f2h(const float* in, uint32_t n, uint32_t dim, uint32_t d8, float alpha, uint4* out, cudaStream_t s) {
    size_t total = (size_t)n * d8;
    unsigned blocks = (unsigned)std::min<size_t>((total + 255) / 256, 148 * 32);
    if (blocks == 0) return;
    f2h_kernel<<<blocks, 256, 0, s>>>(in, n, dim, d8, alpha, reinterpret_cast<__half*>(out));
}

template <typename T>
static gf_status dalloc(T** p, size_t count, uint64_t* bytes) {
    size_t b = std::max<size_t>(count, 1) * sizeof(T);
    cudaError_t e = cudaMalloc((void**)p, b);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc");
    *bytes += b;
    return GF_OK;
}

#define GF_TRY(x)                       \
    do {                                \
        gf_status s_ = (x);             \
        if (s_ != GF_OK) return s_;     \
    } while (0)

static void free_index(DeviceIndex& d) {
    void* ptrs[] = {d.vec16,   d.vec32,   d.attrs,     d.graph,   d.cross,   d.i2g,     d.seg,
                    d.grid_d,  d.lq_d,    d.rq_d,      d.centroids, d.hist,  d.entry,   d.sh_slot,
                    d.sh_gofs, d.sh_xofs, d.sh_vsh,    d.vec8,      d.csc,   d.cbi,     d.cnorm,
                    d.cmean,   d.spk_rank, d.fgraph, d.fentry};
    for (void* p : ptrs)
        if (p) cudaFree(p);
    if (d.graph_h) cudaFreeHost(d.graph_h);
    if (d.cross_h) cudaFreeHost(d.cross_h);
    free_bf_tc(d);
}

// compress_global_graph_extreme (tools.cuh:917-935): positions in cell order; a point that is
// still its own spokesman claims, in its graph row's order, every neighbour of higher position
// that is still its own spokesman.  rank = index of the spokesman among all spokesmen in
// position order (the reference's center_pos, tools.cuh:978-986).
void spokesman_assign(uint32_t n, uint32_t n_cells, const uint32_t* cell_sizes, uint32_t degree,
                      const uint32_t* graphs, uint32_t* spk, uint32_t* rank, uint32_t* n_spk) {
    for (uint32_t i = 0; i < n; ++i) spk[i] = i;
    uint32_t off = 0;
    for (uint32_t c = 0; c < n_cells; ++c) {
        const uint32_t sz = cell_sizes[c];
        for (uint32_t j = 0; j < sz; ++j) {
            const uint32_t i = off + j;
            if (spk[i] != i) continue;
            for (uint32_t k = 0; k < degree; ++k) {
                const uint32_t loc = graphs[(size_t)i * degree + k];
                if (loc >= sz) continue;  // not a point of this cell
                const uint32_t x = off + loc;
                if (spk[x] == x && x > i) spk[x] = i;
            }
        }
        off += sz;
    }
    uint32_t cnt = 0;
    std::vector<uint32_t> r(rank ? 0 : n);
    uint32_t* rk = rank ? rank : r.data();
    for (uint32_t i = 0; i < n; ++i) {
        if (spk[i] == i) rk[i] = cnt++;
        else rk[i] = rk[spk[i]];  // spk[i] < i: its rank is already known
    }
    if (n_spk) *n_spk = cnt;
}

// Deterministic entry local ids: std::mt19937 with its default seed (as the reference,
// gpu_graph.cu:12503-12526), value = draw % range, duplicates skipped, in draw order.
// The reference further shuffles with std::random_shuffle, whose rand() state carries
// over between calls; this sequence is fixed instead.
static std::vector<uint32_t> make_entry(uint32_t count, uint32_t range) {
    std::vector<uint32_t> out;
    if (range == 0) return out;
    count = std::min(count, range);
    std::mt19937 rng;
    std::vector<uint8_t> seen(range, 0);
    while (out.size() < count) {
        uint32_t t = (uint32_t)(rng() % range);
        if (!seen[t]) {
            seen[t] = 1;
            out.push_back(t);
        }
    }
    return out;
}

static gf_status create(const gf_index_desc* ds, int device, gf_index** out) {
    if (!ds || !out) return fail(GF_ERR_ARG, "null argument");
    *out = nullptr;
    if (ds->n == 0 || ds->dim == 0) return fail(GF_ERR_ARG, "empty index");
    if (ds->n > kPosMask) return fail(GF_ERR_ARG, "more than 2^30-1 points");
    if (ds->n_attr == 0 || ds->n_attr > kMaxAttr) return fail(GF_ERR_ARG, "n_attr must be 1..8");
    if (!ds->vectors || !ds->attrs || !ds->grid || !ds->l_quant || !ds->r_quant || !ds->cell_of || !ds->graphs)
        return fail(GF_ERR_ARG, "missing array");
    if (ds->degree == 0 || ds->degree > 256) return fail(GF_ERR_ARG, "degree must be 1..256");
    if (ds->cross_e > 4) return fail(GF_ERR_ARG, "cross_e must be 0..4");
    if (ds->cross_e && !ds->cross) return fail(GF_ERR_ARG, "missing cross edges");
    const bool sharded = ds->shard_cells && ds->n_shard_cells;
    if (ds->codec > 2) return fail(GF_ERR_ARG, "codec must be 0 (fp16), 1 (int8) or 2 (uint8)");
    if (ds->codec == 2 && !ds->codes) return fail(GF_ERR_ARG, "uint8 codec needs codes");
    if (ds->codec == 1 && ds->codes && (!ds->code_scales || !ds->code_zero_points))
        return fail(GF_ERR_ARG, "int8 codes need their scales and zero points");
    if (sharded && (ds->host_graph || ds->keep_fp32))
        return fail(GF_ERR_ARG, "a shard cannot keep host graphs or fp32 vectors");
    if (ds->cross_spokesman && sharded)
        return fail(GF_ERR_ARG, "spokesman-compressed cross edges need a whole index (not a shard)");
    uint64_t ncells = 1, nq = 0;
    for (uint32_t j = 0; j < ds->n_attr; ++j) {
        if (ds->grid[j] == 0) return fail(GF_ERR_ARG, "zero grid size");
        ncells *= ds->grid[j];
        nq += ds->grid[j];
    }
    if (ncells > 65536) return fail(GF_ERR_ARG, "more than 65536 cells");
    if (ds->dim > 4096) return fail(GF_ERR_ARG, "dim > 4096");

    gf_index* ix = new gf_index();
    DeviceIndex& d = ix->d;
    d.device = device;
    d.n = ds->n;
    d.dim = ds->dim;
    d.d8 = (ds->dim + 7) / 8 * 8;
    d.d4 = (ds->dim + 3) / 4 * 4;
    d.a = ds->n_attr;
    d.ncells = (uint32_t)ncells;
    d.degree = ds->degree;
    d.E = ds->cross_e;
    d.alpha = ds->f2h_factor;
    d.grid.assign(ds->grid, ds->grid + ds->n_attr);
    d.lq.assign(ds->l_quant, ds->l_quant + nq);
    d.rq.assign(ds->r_quant, ds->r_quant + nq);

    const uint32_t n = d.n, P = d.ncells, R = d.degree, E = d.E;
    // positions (get_idx_mapper, tools.cuh:862-889)
    d.seg_h.assign(P + 1, 0);
    for (uint32_t i = 0; i < n; ++i) {
        if (ds->cell_of[i] >= P) {
            delete ix;
            return fail(GF_ERR_FORMAT, "cell id out of range at point " + std::to_string(i));
        }
        d.seg_h[ds->cell_of[i] + 1]++;
    }
    uint32_t minc = 0xFFFFFFFFu;
    for (uint32_t c = 0; c < P; ++c) {
        uint32_t sz = d.seg_h[c + 1];
        if (sz && sz < minc) minc = sz;
        d.seg_h[c + 1] += d.seg_h[c];
    }
    d.min_cell = minc == 0xFFFFFFFFu ? 0 : minc;
    std::vector<uint32_t> i2g(n), pos_of(n);
    {
        std::vector<uint32_t> fill(P, 0);
        for (uint32_t i = 0; i < n; ++i) {
            uint32_t c = ds->cell_of[i];
            uint32_t p = d.seg_h[c] + fill[c]++;
            i2g[p] = i;
            pos_of[i] = p;
        }
    }
    d.entry_h = make_entry(std::max<uint32_t>(R, 64), d.min_cell);
    d.host_graph = ds->host_graph != 0;
    d.n_stored = n;
    d.codec = ds->codec;
    d.d16 = (d.dim + 15) / 16 * 16;
    std::vector<int8_t> qcodes;  // int8 codes quantised here (global order)
    if (d.codec) {
        d.scales_h.assign(d.dim, 0.01f);
        d.zps_h.assign(d.dim, 0);
        if (d.codec == 1 && !ds->codes) {
            qcodes.resize((size_t)n * d.dim);
            quantize_i8_host(ds->vectors, n, d.dim, d.alpha, qcodes.data(), d.scales_h.data(), d.zps_h.data());
        } else {
            if (ds->code_scales) d.scales_h.assign(ds->code_scales, ds->code_scales + d.dim);
            if (ds->code_zero_points) d.zps_h.assign(ds->code_zero_points, ds->code_zero_points + d.dim);
        }
    }

    // Graph rows are already in position order; local ids -> positions.  Cross edges:
    // source-major (position, target cell, edge) on the device; with host_graph,
    // target-major (target cell, position, edge) in pinned host memory, so that the block
    // of one (target, source cell) pair is contiguous for the per-batch copies
    // (the transposed layout of big_dataset_adapterV3.cuh:3539-3542).
    std::vector<uint32_t> graph, cross;
    uint32_t* gdst = nullptr;
    uint32_t* xdst = nullptr;
    // spokesman compression (compress_global_graph_extreme, tools.cuh:917-1010): a position
    // reads the cross row of its spokesman's rank; ranks are in position order and a
    // spokesman lies in its points' cell, so the ranks of cell c are spk_start_h[c] ..
    std::vector<uint32_t> spk, spk_rank;
    uint32_t n_spk = n;
    const bool use_spk = ds->cross_spokesman && E;
    if (use_spk) {
        std::vector<uint32_t> sizes(P);
        for (uint32_t c = 0; c < P; ++c) sizes[c] = d.seg_h[c + 1] - d.seg_h[c];
        spk.resize(n);
        spk_rank.resize(n);
        spokesman_assign(n, P, sizes.data(), R, ds->graphs, spk.data(), spk_rank.data(), &n_spk);
        d.spk_start_h.assign(P + 1, 0);
        for (uint32_t p = 0; p < n; ++p)
            if (spk[p] == p) d.spk_start_h[ds->cell_of[i2g[p]] + 1]++;
        for (uint32_t c = 0; c < P; ++c) d.spk_start_h[c + 1] += d.spk_start_h[c];
    }
    // stored rows: every position, or the shard's cells back to back in shard order
    std::vector<uint32_t> row_pos;  // stored row -> position (shard only)
    std::vector<int32_t> sh_slot;
    std::vector<long long> sh_gofs, sh_xofs, sh_vsh;
    if (sharded) {
        const uint32_t S = ds->n_shard_cells;
        d.sharded = true;
        d.shard_cells.assign(ds->shard_cells, ds->shard_cells + S);
        sh_slot.assign(P, -1);
        for (uint32_t b = 0; b < S; ++b) {
            const uint32_t c = d.shard_cells[b];
            if (c >= P || sh_slot[c] >= 0) {
                delete ix;
                return fail(GF_ERR_ARG, "shard cell out of range or repeated");
            }
            sh_slot[c] = (int32_t)b;
        }
        for (uint32_t b = 0; b < S; ++b) {
            const uint32_t c = d.shard_cells[b];
            sh_vsh.push_back((long long)row_pos.size() - d.seg_h[c]);
            sh_gofs.push_back((long long)row_pos.size() * R);
            for (uint32_t p = d.seg_h[c]; p < d.seg_h[c + 1]; ++p) row_pos.push_back(p);
        }
        d.n_stored = (uint32_t)row_pos.size();
        graph.assign((size_t)d.n_stored * R, kEmpty);
        for (size_t r = 0; r < row_pos.size(); ++r) {
            const uint32_t pos = row_pos[r], c = ds->cell_of[i2g[pos]];
            const uint32_t base = d.seg_h[c], sz = d.seg_h[c + 1] - base;
            for (uint32_t j = 0; j < R; ++j) {
                const uint32_t loc = ds->graphs[(size_t)pos * R + j];
                graph[r * R + j] = loc < sz ? base + loc : kEmpty;
            }
        }
        // cross blocks [target slot][source slot]: source rows of the source cell, E each
        sh_xofs.assign((size_t)S * S, 0);
        long long x = 0;
        // cross_row reads xofs[target][source] + source position * E: each entry is the
        // block's start less the source cell's first position times E
        std::vector<long long> xstart((size_t)S * S);
        for (uint32_t bt = 0; bt < S; ++bt)
            for (uint32_t bs = 0; bs < S; ++bs) {
                xstart[(size_t)bt * S + bs] = x;
                sh_xofs[(size_t)bt * S + bs] = x - (long long)d.seg_h[d.shard_cells[bs]] * E;
                x += (long long)(d.seg_h[d.shard_cells[bs] + 1] - d.seg_h[d.shard_cells[bs]]) * E;
            }
        cross.assign(std::max<long long>(x, 1), kEmpty);
        for (uint32_t bt = 0; bt < S && E; ++bt) {
            const uint32_t ct = d.shard_cells[bt], tbase = d.seg_h[ct], tsz = d.seg_h[ct + 1] - tbase;
            for (uint32_t bs = 0; bs < S; ++bs) {
                const uint32_t cs = d.shard_cells[bs];
                uint32_t* dst = cross.data() + xstart[(size_t)bt * S + bs];
                for (uint32_t p = d.seg_h[cs]; p < d.seg_h[cs + 1]; ++p)
                    for (uint32_t j = 0; j < E; ++j) {
                        const uint32_t loc = ds->cross[(size_t)i2g[p] * P * E + (size_t)ct * E + j];
                        dst[(size_t)(p - d.seg_h[cs]) * E + j] = loc < tsz ? tbase + loc : kEmpty;
                    }
            }
        }
    } else if (d.host_graph) {
        DeviceGuard g0(device);
        cudaError_t e = cudaMallocHost((void**)&d.graph_h, std::max<size_t>((size_t)n * R, 1) * 4);
        if (e == cudaSuccess && E)
            e = cudaMallocHost((void**)&d.cross_h, std::max<size_t>((size_t)n_spk * P * E, 1) * 4);
        if (e != cudaSuccess) {
            free_index(d);
            delete ix;
            return cuda_fail(e, "pinned host graph");
        }
        gdst = d.graph_h;
        xdst = d.cross_h;
    } else {
        graph.resize((size_t)n * R);
        gdst = graph.data();
        if (E) {
            cross.resize((size_t)n * P * E);
            xdst = cross.data();
        }
    }
    for (uint32_t c = 0; c < P && !sharded; ++c) {
        uint32_t base = d.seg_h[c], sz = d.seg_h[c + 1] - base;
        for (size_t r = base; r < (size_t)base + sz; ++r)
            for (uint32_t j = 0; j < R; ++j) {
                uint32_t loc = ds->graphs[r * R + j];
                gdst[r * R + j] = loc < sz ? base + loc : kEmpty;
            }
    }
    if (E && !sharded) {
        const size_t rowlen = (size_t)P * E;
        for (uint32_t g = 0; g < n; ++g) {
            const uint32_t* src = ds->cross + (size_t)g * rowlen;
            const size_t pos = pos_of[g];
            if (d.host_graph && use_spk && spk[pos] != pos) continue;  // only spokesmen keep a row
            const size_t hrow = d.host_graph && use_spk ? spk_rank[pos] : pos;
            for (uint32_t c = 0; c < P; ++c) {
                uint32_t base = d.seg_h[c], sz = d.seg_h[c + 1] - base;
                uint32_t* dst = d.host_graph ? xdst + ((size_t)c * n_spk + hrow) * E : xdst + pos * rowlen + (size_t)c * E;
                for (uint32_t j = 0; j < E; ++j) {
                    uint32_t loc = src[c * E + j];
                    dst[j] = loc < sz ? base + loc : kEmpty;
                }
            }
        }
    }
    d.cross_rows = n;
    if (use_spk) {
        d.cross_rows = n_spk;
        if (!d.host_graph) {
            // keep the rows of spokesmen only; a position reads the row of its spokesman's rank
            const size_t rowlen = (size_t)P * E;
            std::vector<uint32_t> comp((size_t)n_spk * rowlen);
            for (uint32_t p = 0; p < n; ++p)
                if (spk[p] == p)
                    std::memcpy(&comp[(size_t)spk_rank[p] * rowlen], &cross[(size_t)p * rowlen], rowlen * 4);
            cross.swap(comp);
        }
    }
    std::vector<float> attrs((size_t)n * d.a);
    for (uint32_t p = 0; p < n; ++p)
        std::memcpy(&attrs[(size_t)p * d.a], ds->attrs + (size_t)i2g[p] * d.a, sizeof(float) * d.a);
    // Do the cells hold their rows?  Every (numeric) attribute of a row must lie in the
    // closed range [l_quant, r_quant] of its cell's slice in that dimension; cell ids are
    // mixed radix over the slices, last dimension fastest (indexbuild/tools.py:112-120).
    // Only then is "every in-box row of the index" the same set as "every in-box row of
    // the cells the box meets" (the reference's exact route scans the query's cells,
    // gpu_graph.cu:3788-4022), which lets the search find exact-route rows through the
    // attribute tiles.  cell_of comes from the caller, and the reference's quantiles are
    // integers (real_dataset_adapter.cuh:578), so fractional attributes can fall between
    // two slices; such an index keeps the cell scan.
    d.cells_hold_rows = true;
    {
        std::vector<uint32_t> goff(d.a, 0);
        for (uint32_t j = 1; j < d.a; ++j) goff[j] = goff[j - 1] + d.grid[j - 1];
        std::vector<uint32_t> sl(d.a);
        for (uint32_t c = 0; c < P && d.cells_hold_rows; ++c) {
            uint32_t rest = c;
            for (uint32_t j = d.a; j-- > 0;) {
                sl[j] = goff[j] + rest % d.grid[j];
                rest /= d.grid[j];
            }
            for (uint32_t p = d.seg_h[c]; p < d.seg_h[c + 1] && d.cells_hold_rows; ++p)
                for (uint32_t j = 0; j < d.a; ++j) {
                    const float v = attrs[(size_t)p * d.a + j];
                    if (v < d.lq[sl[j]] || v > d.rq[sl[j]]) {  // NaN rows are in no box: they pass
                        d.cells_hold_rows = false;
                        break;
                    }
                }
        }
    }

    // clusters (load_clustering, tools.cuh:569-602): centroid = float mean accumulated in
    // global point order; hist[cell][label]
    std::vector<float> centroids;
    std::vector<uint32_t> hist;
    if (ds->n_clusters && ds->labels) {
        int32_t mx = -1;
        for (uint32_t i = 0; i < n; ++i) {
            if (ds->labels[i] < 0) {
                free_index(d);
                delete ix;
                return fail(GF_ERR_FORMAT, "negative cluster label");
            }
            mx = std::max(mx, ds->labels[i]);
        }
        d.C = (uint32_t)(mx + 1);
        centroids.assign((size_t)d.C * d.dim, 0.0f);
        hist.assign((size_t)P * d.C, 0);
        std::vector<uint32_t> num(d.C, 0);
        for (uint32_t i = 0; i < n; ++i) {
            uint32_t c = (uint32_t)ds->labels[i];
            num[c]++;
            hist[(size_t)ds->cell_of[i] * d.C + c]++;
            float* cr = &centroids[(size_t)c * d.dim];
            const float* v = ds->vectors + (size_t)i * d.dim;
            for (uint32_t k = 0; k < d.dim; ++k) cr[k] += v[k];
        }
        for (uint32_t c = 0; c < d.C; ++c)
            for (uint32_t k = 0; k < d.dim; ++k) centroids[(size_t)c * d.dim + k] /= (float)num[c];
    }
    // tensor-core planner inputs: the centroids' mean m and, per centroid, the squared norm
    // of c - m (fp32 differences, as the device forms them) and its square root
    std::vector<float> cmean(d.C ? d.dim : 0, 0.0f), cnorm(2 * (size_t)d.C, 0.0f);
    if (d.C) {
        // mean over the finite centroids (an empty cluster's centroid is 0/0)
        std::vector<double> msum(d.dim, 0.0);
        uint32_t nfin = 0;
        for (uint32_t c = 0; c < d.C; ++c) {
            const float* cr = &centroids[(size_t)c * d.dim];
            bool fin = true;
            for (uint32_t k = 0; k < d.dim && fin; ++k) fin = std::isfinite(cr[k]);
            if (!fin) continue;
            ++nfin;
            for (uint32_t k = 0; k < d.dim; ++k) msum[k] += cr[k];
        }
        for (uint32_t k = 0; k < d.dim; ++k) cmean[k] = nfin ? (float)(msum[k] / nfin) : 0.0f;
        for (uint32_t c = 0; c < d.C; ++c) {
            float acc = 0.0f;
            for (uint32_t k = 0; k < d.dim; ++k) {
                const float t = centroids[(size_t)c * d.dim + k] - cmean[k];
                acc += t * t;
            }
            cnorm[2 * (size_t)c] = acc;
            cnorm[2 * (size_t)c + 1] = std::sqrt(acc);
        }
    }

    DeviceGuard guard(device);
    gf_status st = GF_OK;
    auto chk = [&](gf_status s) {
        if (st == GF_OK && s != GF_OK) st = s;
        return st == GF_OK;
    };
    float* vtmp = nullptr;
    do {
        const uint32_t nrows = sharded ? d.n_stored : n;
        if (!d.codec && !chk(dalloc(&d.vec16, (size_t)nrows * d.d8 / 8, &d.bytes))) break;
        if (d.codec) {
            if (!chk(dalloc(&d.vec8, (size_t)nrows * d.d16 / 16, &d.bytes))) break;
            if (!chk(dalloc(&d.csc, d.d16, &d.bytes))) break;
            if (!chk(dalloc(&d.cbi, d.d16, &d.bytes))) break;
            // byte rows in stored order, zero padded; scale 0 past dim decodes padding to 0
            const uint8_t* codes = ds->codes ? ds->codes : reinterpret_cast<const uint8_t*>(qcodes.data());
            std::vector<uint8_t> rows8((size_t)nrows * d.d16, 0);
            for (size_t r = 0; r < nrows; ++r) {
                const uint32_t pos = sharded ? row_pos[r] : (uint32_t)r;
                std::memcpy(&rows8[r * d.d16], codes + (size_t)i2g[pos] * d.dim, d.dim);
            }
            std::vector<float> sc(d.d16, 0.0f), bi(d.d16, 8388608.0f);  // sc holds -scale
            for (uint32_t j = 0; j < d.dim; ++j) {
                sc[j] = -d.scales_h[j];
                bi[j] = 8388608.0f + (float)(d.zps_h[j] + (d.codec == 1 ? 128 : 0));
            }
            cudaError_t e = cudaMemcpy(d.vec8, rows8.data(), rows8.size(), cudaMemcpyHostToDevice);
            if (e == cudaSuccess) e = cudaMemcpy(d.csc, sc.data(), sc.size() * 4, cudaMemcpyHostToDevice);
            if (e == cudaSuccess) e = cudaMemcpy(d.cbi, bi.data(), bi.size() * 4, cudaMemcpyHostToDevice);
            if (e != cudaSuccess) {
                st = cuda_fail(e, "upload byte rows");
                break;
            }
        }
        if (!chk(dalloc(&d.attrs, (size_t)n * d.a, &d.bytes))) break;
        if (!d.host_graph && !chk(dalloc(&d.graph, graph.size(), &d.bytes))) break;
        if (!d.host_graph && E && !chk(dalloc(&d.cross, cross.size(), &d.bytes))) break;
        if (!spk_rank.empty() && !chk(dalloc(&d.spk_rank, spk_rank.size(), &d.bytes))) break;
        if (sharded) {
            if (!chk(dalloc(&d.sh_slot, sh_slot.size(), &d.bytes))) break;
            if (!chk(dalloc(&d.sh_gofs, sh_gofs.size(), &d.bytes))) break;
            if (!chk(dalloc(&d.sh_xofs, sh_xofs.size(), &d.bytes))) break;
            if (!chk(dalloc(&d.sh_vsh, sh_vsh.size(), &d.bytes))) break;
        }
        if (!chk(dalloc(&d.i2g, n, &d.bytes))) break;
        if (!chk(dalloc(&d.seg, P + 1, &d.bytes))) break;
        if (!chk(dalloc(&d.grid_d, d.a, &d.bytes))) break;
        if (!chk(dalloc(&d.lq_d, nq, &d.bytes))) break;
        if (!chk(dalloc(&d.rq_d, nq, &d.bytes))) break;
        if (!chk(dalloc(&d.entry, d.entry_h.size(), &d.bytes))) break;
        if (d.C) {
            if (!chk(dalloc(&d.centroids, (size_t)d.C * d.dim, &d.bytes))) break;
            if (!chk(dalloc(&d.hist, (size_t)P * d.C, &d.bytes))) break;
            if (!chk(dalloc(&d.cnorm, 2 * (size_t)d.C, &d.bytes))) break;
            if (!chk(dalloc(&d.cmean, d.dim, &d.bytes))) break;
        }
        // fp32 rows in position order (temporary unless kept)
        uint64_t dummy = 0;
        if (ds->keep_fp32) {
            if (!chk(dalloc(&d.vec32, (size_t)n * d.d4 / 4, &d.bytes))) break;
        }
        const bool need_f32 = !d.codec || d.vec32;  // fp16 conversion or kept fp32 rows
        if (need_f32 && !chk(dalloc(&vtmp, (size_t)nrows * d.dim, &dummy))) break;
        std::vector<float> rows((size_t)std::min<uint32_t>(std::max<uint32_t>(nrows, 1), 65536) * d.dim);
        const uint32_t chunk = std::min<uint32_t>(std::max<uint32_t>(nrows, 1), 65536);
        for (uint32_t p0 = 0; need_f32 && p0 < nrows && st == GF_OK; p0 += chunk) {
            uint32_t cnt = std::min(chunk, nrows - p0);
            for (uint32_t r = 0; r < cnt; ++r) {
                const uint32_t pos = sharded ? row_pos[p0 + r] : p0 + r;
                std::memcpy(&rows[(size_t)r * d.dim], ds->vectors + (size_t)i2g[pos] * d.dim, sizeof(float) * d.dim);
            }
            cudaError_t e = cudaMemcpy(vtmp + (size_t)p0 * d.dim, rows.data(), sizeof(float) * cnt * d.dim,
                                       cudaMemcpyHostToDevice);
            if (e != cudaSuccess) st = cuda_fail(e, "upload vectors");
        }
        if (st != GF_OK) break;
        if (nrows && !d.codec) launch_f2h(vtmp, nrows, d.dim, d.d8, d.alpha, d.vec16, 0);
        if (d.vec32) {
            cudaError_t e = cudaMemset2D(d.vec32, sizeof(float) * d.d4, 0, sizeof(float) * d.d4, n);
            if (e == cudaSuccess)
                e = cudaMemcpy2D(d.vec32, sizeof(float) * d.d4, vtmp, sizeof(float) * d.dim, sizeof(float) * d.dim,
                                 n, cudaMemcpyDeviceToDevice);
            if (e != cudaSuccess) {
                st = cuda_fail(e, "fp32 rows");
                break;
            }
        }
        struct Up {
            void* dst;
            const void* src;
            size_t bytes;
        } ups[] = {
            {d.attrs, attrs.data(), attrs.size() * 4},
            {d.graph, graph.data(), graph.size() * 4},
            {d.cross, cross.data(), cross.size() * 4},
            {d.spk_rank, spk_rank.data(), spk_rank.size() * 4},
            {d.i2g, i2g.data(), i2g.size() * 4},
            {d.seg, d.seg_h.data(), d.seg_h.size() * 4},
            {d.grid_d, d.grid.data(), d.grid.size() * 4},
            {d.lq_d, d.lq.data(), d.lq.size() * 4},
            {d.rq_d, d.rq.data(), d.rq.size() * 4},
            {d.entry, d.entry_h.data(), d.entry_h.size() * 4},
            {d.centroids, centroids.data(), centroids.size() * 4},
            {d.hist, hist.data(), hist.size() * 4},
            {d.cnorm, cnorm.data(), cnorm.size() * 4},
            {d.cmean, cmean.data(), cmean.size() * 4},
            {d.sh_slot, sh_slot.data(), sh_slot.size() * 4},
            {d.sh_gofs, sh_gofs.data(), sh_gofs.size() * 8},
            {d.sh_xofs, sh_xofs.data(), sh_xofs.size() * 8},
            {d.sh_vsh, sh_vsh.data(), sh_vsh.size() * 8},
        };
        for (auto& u : ups) {
            if (!u.dst || u.bytes == 0) continue;
            cudaError_t e = cudaMemcpy(u.dst, u.src, u.bytes, cudaMemcpyHostToDevice);
            if (e != cudaSuccess) {
                st = cuda_fail(e, "upload index");
                break;
            }
        }
        if (st != GF_OK) break;
        if ((st = attr_tiles_prepare(d)) != GF_OK) break;        // attribute tiles (box counts, brute force)
        if (d.vec32 && (st = bf_tc_prepare(d)) != GF_OK) break;  // fp16 tiles of the tensor-core brute force
        cudaError_t e = cudaDeviceSynchronize();
        if (e == cudaSuccess) e = cudaGetLastError();
        if (e != cudaSuccess) st = cuda_fail(e, "index build");
    } while (0);
    if (vtmp) cudaFree(vtmp);
    if (st != GF_OK) {
        free_index(d);
        delete ix;
        return st;
    }
    *out = ix;
    return GF_OK;
}

}  // namespace gf

using namespace gf;

extern "C" {

const char* gf_status_string(gf_status s) {
    switch (s) {
        case GF_OK: return "ok";
        case GF_ERR_ARG: return "invalid argument";
        case GF_ERR_IO: return "i/o error";
        case GF_ERR_FORMAT: return "format error";
        case GF_ERR_OOM: return "out of memory";
        case GF_ERR_CUDA: return "cuda error";
        case GF_ERR_TIMEOUT: return "timeout";
        case GF_ERR_STATE: return "bad call order";
    }
    return "unknown status";
}

const char* gf_last_error(void) { return g_err.c_str(); }

const char* gf_version(void) { return "garfield_b200 0.1 (sm_100a)"; }

void gf_search_defaults(gf_search_params* p) {
    if (!p) return;
    p->L = 64;
    p->k = 10;
    p->width = 1;
    p->max_iter = 10000;
    p->n_entry = 0;  // 0 = graph degree
    p->postfilter = 0xFFFFFFFFu;
    p->hash_slots = 0;
    p->test_wait = 0;
    p->exact_tc = 0;
    p->route = 0;
}

gf_status gf_index_create(const gf_index_desc* desc, int device, gf_index** out) {
    return create(desc, device, out);
}

gf_status gf_index_info_get(const gf_index* idx, gf_index_info* out) {
    if (!idx || !out) return fail(GF_ERR_ARG, "null argument");
    const DeviceIndex& d = idx->d;
    out->n = d.n;
    out->dim = d.dim;
    out->n_attr = d.a;
    out->n_cells = d.ncells;
    out->degree = d.degree;
    out->cross_e = d.E;
    out->n_clusters = d.C;
    out->d_stored = d.d8;
    out->min_cell_size = d.min_cell;
    out->cross_rows = d.cross_rows;
    out->device_bytes = d.bytes;
    return GF_OK;
}

gf_status gf_index_entry_points(const gf_index* idx, uint32_t n, uint32_t* out_host) {
    if (!idx || !out_host) return fail(GF_ERR_ARG, "null argument");
    if (n > idx->d.entry_h.size()) return fail(GF_ERR_ARG, "more entry points than available");
    std::memcpy(out_host, idx->d.entry_h.data(), sizeof(uint32_t) * n);
    return GF_OK;
}

gf_status gf_index_destroy(gf_index* idx) {
    if (!idx) return GF_OK;
    DeviceGuard guard(idx->d.device);
    free_index(idx->d);
    delete idx;
    return GF_OK;
}

}  // extern "C"
