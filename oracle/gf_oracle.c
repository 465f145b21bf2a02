/*
 * gf_oracle.c -- CPU restatement of the Garfield GMG query path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker the CUDA product is compared
 * against; it is never linked into the product library and no product code path
 * calls it.  Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg
 * load it.
 *
 * Every function restates one piece of the reference (ZJU-DAILY/Garfield,
 * indexsearch/) in plain C with a fixed floating-point evaluation order, so that the
 * CUDA kernels, which use the same order, can be compared bit-exactly:
 *
 *   orc_f2h            tools.cuh:308-321               f2h(data, half, n, D, alpha)
 *   orc_bruteforce     gpu_graph.cu:10782-10812        naive_brute_force_with_filter
 *   orc_plan_cells     real_dataset_adapter.cuh:127-213 + 390-519
 *                                                      intersection_area_..._closed_interval
 *                                                      + thrust copy_if/reduce_by_key/scan CSR
 *   orc_count_in_box   real_dataset_adapter.cuh:347-387 prefiltering_tag_elements
 *   orc_order_cells    tools.cuh:1399-1586, gpu_graph.cu:11344-11396,11742-11845
 *                                                      dis_cal_tensor_core + select_topk_by_reduce_min
 *                                                      + sort_by_clustering_info_weighted
 *   orc_cluster_info   tools.cuh:569-602               load_clustering (centroids, histogram)
 *   orc_search         gpu_graph.cu:3270-4131          select_path_contain_attr_filter_V2_
 *                                                      without_output_with_post_pre_filter
 *   orc_recall         tools.cuh:456-544               cal_recall_show_partition_multi_attrs
 *   orc_quantize_i8    production_adapter.cuh:316-337  per-dimension affine int8 codec (host path of
 *                                                      load_dataset_return_int8_arr_infile)
 *   orc_dist8          big_dataset_adapterV3.cuh:852-863, 2802-2810  distances to int8 / uint8 rows
 *   orc_spokesman      tools.cuh:917-935, 978-986      spokesman assignment of the cross-edge
 *                                                      compression (compress_global_graph_extreme)
 *   orc_assemble       full_graph_search.cuh:984-997   assemble_edges (the full-graph ablation's graph)
 *   orc_search_fullgraph full_graph_search.cuh:179-593 full_graph_search_postfiltering
 *
 * Fixed evaluation orders ("canonical distances"), shared with the CUDA kernels:
 *   - orc_dist32: squared L2 of two rows of padded length (a multiple of 4).  Eight
 *     partial sums: element i feeds p[i mod 8], in increasing order of i, with one fused
 *     multiply-add p = fma(q-x, q-x, p) (q-x rounded to fp32 first).  Then
 *     s[j] = p[j] + p[j+4] (j<4), t[j] = s[j] + s[j+2] (j<2), result = t[0] + t[1] ("finish8").
 *     (Adjacent partials are the two halves of one packed two-wide fp32 register on the
 *     GPU, so every step is one packed instruction and the chunk loop needs no unrolling.)
 *   - orc_dist16 (search rows, fp16): the row is cut into 16-byte chunks of 8 elements;
 *     chunks of even index feed partial set 0, odd chunks set 1, element i feeding
 *     p[set][i mod 8] as above; then s[j] = p[0][j] + p[1][j] and finish8(s).  (On the GPU
 *     two lanes share a row, one per chunk parity, and add their partials once.)
 *   - orc_dist8: the same two partial sets over byte rows (d16 elements, 16-element
 *     chunks, set = chunk index mod 2): diff =
 *     fma(-scale[i], (float)(row[i] ^ xmask) - bias[i], q[i]), i.e. q - scale * (code -
 *     bias) with one rounding (the integer difference is exact); q is the fp32 query times
 *     f2h_factor (not rounded to fp16).
 *   - orc_dist_seq: squared L2 with one fma chain over d = 0..D-1 (used for the
 *     query-centroid distances of the cell ordering).
 * The reference accumulates candidate distances in fp16 (gpu_graph.cu:3394-3403) and
 * centroid products with fp16 WMMA (tools.cuh:1512-1537); this restatement and the
 * CUDA port both accumulate in fp32, so results agree with the reference on recall,
 * not on bit patterns.
 *
 * Deterministic choices where the reference is racy or unordered (each mirrored by
 * the CUDA port):
 *   - all candidate lists are ordered by (distance, position) where position is the
 *     point's cell-major "logical position" seg_start[cell] + local id (the
 *     reference's offset[pid] + local_idx, tools.cuh:862-889);
 *   - the brute-force top-k orders by (distance, global id) (lower id wins ties);
 *   - cells of equal score keep increasing cell-id order;
 *   - the cross-cell hop takes the distinct cross-edge targets of the first 64 list
 *     entries plus the smallest unused local ids of the next cell as filler
 *     (gpu_graph.cu:3564-3631 does the same with racing atomics);
 *   - a point is never evaluated twice inside one cell except when the evaluation
 *     cannot change the lists (see orc_search).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_EMPTY 0xFFFFFFFFu
#define ORC_EXPLORED 0x80000000u
#define ORC_INRANGE 0x40000000u
#define ORC_POSMASK 0x3FFFFFFFu

/* ------------------------------------------------------------------ fp16 */

static inline uint16_t f32_to_f16_bits(float x) {
    _Float16 h = (_Float16)x; /* IEEE round-to-nearest-even, as __float2half */
    uint16_t b;
    memcpy(&b, &h, 2);
    return b;
}

static inline float f16_bits_to_f32(uint16_t b) {
    _Float16 h;
    memcpy(&h, &b, 2);
    return (float)h;
}

/* tools.cuh:308-321: half(x * alpha), row-major; rows padded with zeros to d_pad. */
void orc_f2h(const float* in, uint32_t n, uint32_t dim, uint32_t d_pad, float alpha, uint16_t* out) {
    for (size_t i = 0; i < (size_t)n; ++i) {
        for (uint32_t d = 0; d < d_pad; ++d) {
            float v = d < dim ? in[i * dim + d] * alpha : 0.0f;
            out[i * d_pad + d] = f32_to_f16_bits(v);
        }
    }
}

/* ----------------------------------------------------- canonical distances */

static inline float finish8(const float p[8]) {
    float s[4], t[2];
    for (int j = 0; j < 4; ++j) s[j] = p[j] + p[j + 4];
    for (int j = 0; j < 2; ++j) t[j] = s[j] + s[j + 2];
    return t[0] + t[1];
}

/* fp16 rows of d8 elements (d8 % 8 == 0): two partial sets by chunk parity. */
float orc_dist16(const uint16_t* q, const uint16_t* x, uint32_t d8) {
    float p[2][8] = {{0}};
    for (uint32_t i = 0; i < d8; ++i) {
        float diff = f16_bits_to_f32(q[i]) - f16_bits_to_f32(x[i]);
        float* ps = p[(i / 8) & 1];
        ps[i & 7] = fmaf(diff, diff, ps[i & 7]);
    }
    float s8[8];
    for (int j = 0; j < 8; ++j) s8[j] = p[0][j] + p[1][j];
    return finish8(s8);
}

/* fp32 rows of d4 elements (d4 % 4 == 0). */
float orc_dist32(const float* q, const float* x, uint32_t d4) {
    float p[8] = {0};
    for (uint32_t i = 0; i < d4; ++i) {
        float diff = q[i] - x[i];
        p[i & 7] = fmaf(diff, diff, p[i & 7]);
    }
    return finish8(p);
}

/* byte rows of d16 elements; see the header for the formula */
float orc_dist8(const float* q, const uint8_t* x, const float* scale, const float* bias, uint32_t xmask,
                uint32_t d16) {
    float p[2][8] = {{0}};
    for (uint32_t i = 0; i < d16; ++i) {
        float diff = fmaf(-scale[i], (float)(uint32_t)(x[i] ^ (uint8_t)xmask) - bias[i], q[i]);
        float* ps = p[(i / 16) & 1];
        ps[i & 7] = fmaf(diff, diff, ps[i & 7]);
    }
    float s8[8];
    for (int j = 0; j < 8; ++j) s8[j] = p[0][j] + p[1][j];
    return finish8(s8);
}

/*
 * Per-dimension affine int8 quantisation, production_adapter.cuh:316-337 (the host path
 * used with a .q file): x = data * alpha; per dimension min / max over all points starting
 * from min = 100000, max = -100000 (as the reference); scale = (max - min) / 255;
 * zero_point = round(-128 - min / scale) clamped to [-128, 127]; q = round(x / scale) +
 * zero_point clamped to [-128, 127]; round = half away from zero (C round).  Where max ==
 * min the reference divides by zero; here scale = 1 for such a dimension.
 */
void orc_quantize_i8(const float* data, uint32_t n, uint32_t dim, float alpha, int8_t* q, float* scales,
                     int32_t* zero_points) {
    for (uint32_t j = 0; j < dim; ++j) {
        float mn = 100000.0f, mx = -100000.0f;
        for (uint32_t i = 0; i < n; ++i) {
            float x = data[(size_t)i * dim + j] * alpha;
            mn = fminf(mn, x);
            mx = fmaxf(mx, x);
        }
        float scale = (mx - mn) / 255.0f;
        if (!(scale > 0.0f)) scale = 1.0f;
        int zp = (int)roundf(-128.0f - mn / scale);
        zp = zp < -128 ? -128 : zp > 127 ? 127 : zp;
        for (uint32_t i = 0; i < n; ++i) {
            float x = data[(size_t)i * dim + j] * alpha;
            int v = (int)roundf(x / scale) + zp;
            v = v < -128 ? -128 : v > 127 ? 127 : v;
            q[(size_t)i * dim + j] = (int8_t)v;
        }
        scales[j] = scale;
        zero_points[j] = zp;
    }
}

float orc_dist_seq(const float* q, const float* x, uint32_t dim) {
    float acc = 0.0f;
    for (uint32_t d = 0; d < dim; ++d) {
        float diff = q[d] - x[d];
        acc = fmaf(diff, diff, acc);
    }
    return acc;
}

/* --------------------------------------------------------------- filters */

static inline int in_box(const float* attr, const float* lb, const float* rb, uint32_t a) {
    for (uint32_t j = 0; j < a; ++j)
        if (!(attr[j] >= lb[j] && attr[j] <= rb[j])) return 0;
    return 1;
}

/* real_dataset_adapter.cuh:347-387: number of points inside each query box. */
void orc_count_in_box(const float* attrs, uint32_t n, uint32_t a, const float* lb, const float* rb,
                      uint32_t qnum, uint32_t* counts) {
#pragma omp parallel for schedule(dynamic, 4)
    for (long q = 0; q < (long)qnum; ++q) {
        uint32_t c = 0;
        for (uint32_t i = 0; i < n; ++i) c += (uint32_t)in_box(attrs + (size_t)i * a, lb + q * a, rb + q * a, a);
        counts[q] = c;
    }
}

/* ------------------------------------------------------ exact filtered scan */

typedef struct {
    float d;
    uint32_t id;
} orc_pair;

/* (distance, id) order; a NaN distance (the 0/0 centroid of an empty cluster, as
 * load_clustering tools.cuh:600-603 computes it) ranks after every number, NaNs by id --
 * the order of the device keys, whose NaN bit pattern is above +inf. */
static inline int pair_less(orc_pair x, orc_pair y) {
    const int xn = isnan(x.d), yn = isnan(y.d);
    if (xn || yn) return xn ? (yn && x.id < y.id) : 1;
    return x.d < y.d || (x.d == y.d && x.id < y.id);
}

/* Insert into a sorted list of capacity k holding *n items; keeps the k smallest. */
static inline void topk_insert(orc_pair* list, uint32_t* n, uint32_t k, orc_pair v) {
    if (*n == k && !pair_less(v, list[k - 1])) return;
    uint32_t i = (*n < k) ? (*n)++ : k - 1;
    while (i > 0 && pair_less(v, list[i - 1])) {
        list[i] = list[i - 1];
        --i;
    }
    list[i] = v;
}

/*
 * gpu_graph.cu:10782-10812 naive_brute_force_with_filter: every point whose attributes
 * lie in the closed box competes; squared distance by orc_dist32 on rows padded to d4;
 * the k smallest (distance, global id).  The reference returns sqrt distances in
 * max-heap pop order; the order here is ascending and the distance is squared.
 * Missing entries (fewer than k points in the box) are ORC_EMPTY / INFINITY.
 */
void orc_bruteforce(const float* data4, uint32_t n, uint32_t d4, const float* attrs, uint32_t a,
                    const float* queries4, const float* lb, const float* rb, uint32_t qnum, uint32_t k,
                    uint32_t* ids_out, float* dist_out, int threads) {
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#endif
#pragma omp parallel
    {
        orc_pair* list = (orc_pair*)malloc(sizeof(orc_pair) * (k ? k : 1));
#pragma omp for schedule(dynamic, 1)
        for (long q = 0; q < (long)qnum; ++q) {
            uint32_t cnt = 0;
            const float* qv = queries4 + (size_t)q * d4;
            for (uint32_t i = 0; i < n; ++i) {
                if (!in_box(attrs + (size_t)i * a, lb + q * a, rb + q * a, a)) continue;
                orc_pair v = {orc_dist32(qv, data4 + (size_t)i * d4, d4), i};
                if (k) topk_insert(list, &cnt, k, v);
            }
            for (uint32_t j = 0; j < k; ++j) {
                ids_out[q * k + j] = j < cnt ? list[j].id : ORC_EMPTY;
                dist_out[q * k + j] = j < cnt ? list[j].d : INFINITY;
            }
        }
        free(list);
    }
}

/* ------------------------------------------------- cross-edge compression */

/*
 * tools.cuh:917-935, 978-986 (compress_global_graph_extreme): spokesman of every position
 * (cells in order, sizes[c] points each, graph rows in position order holding local ids).
 * Scanning positions in order, a point that is still its own spokesman makes every
 * neighbour k of its row (in row order) with position > its own and still its own spokesman
 * a follower.  rank[p] = number of spokesmen at positions before p's spokesman.  Returns
 * the number of spokesmen.
 */
uint32_t orc_spokesman(const uint32_t* sizes, uint32_t ncells, const uint32_t* graphs, uint32_t degree, uint32_t* spk,
                       uint32_t* rank) {
    uint32_t n = 0;
    for (uint32_t c = 0; c < ncells; ++c) n += sizes[c];
    for (uint32_t i = 0; i < n; ++i) spk[i] = i;
    uint32_t off = 0;
    for (uint32_t c = 0; c < ncells; ++c) {
        for (uint32_t j = 0; j < sizes[c]; ++j) {
            const uint32_t i = off + j;
            if (spk[i] != i) continue;
            for (uint32_t k = 0; k < degree; ++k) {
                const uint32_t loc = graphs[(size_t)i * degree + k];
                if (loc >= sizes[c]) continue;
                const uint32_t x = off + loc;
                if (spk[x] == x && x > i) spk[x] = i;
            }
        }
        off += sizes[c];
    }
    uint32_t cnt = 0;
    for (uint32_t i = 0; i < n; ++i) rank[i] = spk[i] == i ? cnt++ : rank[spk[i]];
    return cnt;
}

/* ------------------------------------------------------------- planning */

/*
 * real_dataset_adapter.cuh:127-213 (closed-interval cell intersection) and :390-519
 * (CSR).  Per dimension j the selected slices are s_lo = first s with r_quant[s] >= l
 * (to_lower_bound_linear_scan over r_quant) and s_hi = last s with l_quant[s] <= r
 * (to_upper_bound_linear_scan over l_quant, minus one).  The cells are all mixed-radix
 * combinations, cell id = sum_j idx_j * prod_{k>j} grid_k (gpu_graph.cu:10965-10973),
 * listed in increasing cell id (the order copy_if leaves them in).  A dimension whose
 * range selects no slice gives the query no cells (the reference would still mark one
 * out-of-range cell).  Returns the total number of cells, or -1 if it exceeds cap.
 */
long orc_plan_cells(const float* lb, const float* rb, uint32_t qnum, uint32_t a, const uint32_t* grid,
                    const float* lq, const float* rq, uint32_t* counts, uint32_t* offsets, uint32_t* cells,
                    uint64_t cap) {
    uint64_t total = 0;
    uint32_t npart = 1;
    for (uint32_t j = 0; j < a; ++j) npart *= grid[j];
    uint8_t* sel = (uint8_t*)malloc(npart ? npart : 1);
    for (uint32_t q = 0; q < qnum; ++q) {
        uint32_t off = 0, lo[16], hi[16];
        int empty = 0;
        for (uint32_t j = 0; j < a; ++j) {
            const float* L = lq + off;
            const float* R = rq + off;
            uint32_t g = grid[j], s;
            for (s = 0; s < g && R[s] < lb[q * a + j]; ++s) {
            }
            lo[j] = s;
            for (s = 0; s < g && L[s] <= rb[q * a + j]; ++s) {
            }
            if (s == 0 || lo[j] >= g || s - 1 < lo[j]) empty = 1;
            hi[j] = s - 1;
            off += g;
        }
        memset(sel, 0, npart);
        uint32_t cnt = 0;
        if (!empty) {
            uint32_t idx[16];
            for (uint32_t j = 0; j < a; ++j) idx[j] = lo[j];
            for (;;) {
                uint32_t pid = 0, f = 1;
                for (int j = (int)a - 1; j >= 0; --j) {
                    pid += idx[j] * f;
                    f *= grid[j];
                }
                sel[pid] = 1;
                uint32_t pos = 0;
                while (pos < a) {
                    if (++idx[pos] <= hi[pos]) break;
                    idx[pos] = lo[pos];
                    ++pos;
                }
                if (pos >= a) break;
            }
        }
        offsets[q] = (uint32_t)total;
        for (uint32_t p = 0; p < npart; ++p)
            if (sel[p]) {
                if (total + cnt >= cap) {
                    free(sel);
                    return -1;
                }
                cells[total + cnt++] = p;
            }
        counts[q] = cnt;
        total += cnt;
    }
    free(sel);
    return (long)total;
}

/*
 * tools.cuh:569-602 load_clustering: centroid = float mean of the fp32 rows of each
 * label, accumulated in global point order; histogram hist[cell * C + label] counts the
 * points of each cell (the reference takes cell = i / 62500, which equals the grid
 * cell for cell-contiguous data; here the grid cell of each point is used).
 * C = max label + 1.
 */
void orc_cluster_info(const float* data, uint32_t n, uint32_t dim, const int32_t* labels,
                      const uint32_t* cell_of, uint32_t ncells, uint32_t C, float* centroids, uint32_t* hist) {
    uint32_t* num = (uint32_t*)calloc(C, sizeof(uint32_t));
    memset(centroids, 0, sizeof(float) * (size_t)C * dim);
    memset(hist, 0, sizeof(uint32_t) * (size_t)C * ncells);
    for (size_t i = 0; i < n; ++i) {
        uint32_t c = (uint32_t)labels[i];
        num[c]++;
        hist[(size_t)cell_of[i] * C + c]++;
        for (uint32_t d = 0; d < dim; ++d) centroids[(size_t)c * dim + d] += data[i * dim + d];
    }
    for (uint32_t c = 0; c < C; ++c)
        for (uint32_t d = 0; d < dim; ++d) centroids[(size_t)c * dim + d] /= (float)num[c];
    free(num);
}

/*
 * Cell ordering (tools.cuh:1494-1586, gpu_graph.cu:11344-11396, 11742-11845):
 * the 4 centroids nearest to the query (orc_dist_seq on fp32, ties by centroid id),
 * score(cell) = sum over those 4 of hist[cell][centroid], cells sorted by decreasing
 * score, ties by increasing cell id.  `cells` is reordered in place; the 4 centroid ids
 * of each query are written to top4 (ORC_EMPTY where C < 4).  The reference's
 * "all-little" penalty term is always zero on its live path (the flag array it reads
 * is never set), so it is omitted.
 */
void orc_order_cells(const float* queries, uint32_t qnum, uint32_t dim, const float* centroids, uint32_t C,
                     const uint32_t* hist, const uint32_t* counts, const uint32_t* offsets, uint32_t* cells,
                     uint32_t* top4) {
#pragma omp parallel for schedule(dynamic, 16)
    for (long q = 0; q < (long)qnum; ++q) {
        orc_pair best[4];
        uint32_t nb = 0;
        for (uint32_t c = 0; c < C; ++c) {
            orc_pair v = {orc_dist_seq(queries + (size_t)q * dim, centroids + (size_t)c * dim, dim), c};
            topk_insert(best, &nb, 4, v);
        }
        for (uint32_t t = 0; t < 4; ++t) top4[q * 4 + t] = t < nb ? best[t].id : ORC_EMPTY;
        uint32_t m = counts[q], *cl = cells + offsets[q];
        int64_t* score = (int64_t*)malloc(sizeof(int64_t) * (m ? m : 1));
        for (uint32_t i = 0; i < m; ++i) {
            int64_t s = 0;
            for (uint32_t t = 0; t < nb; ++t) s += hist[(size_t)cl[i] * C + best[t].id];
            score[i] = s;
        }
        /* insertion sort: score desc, cell id asc */
        for (uint32_t i = 1; i < m; ++i) {
            uint32_t c = cl[i];
            int64_t s = score[i];
            uint32_t j = i;
            while (j > 0 && (score[j - 1] < s || (score[j - 1] == s && cl[j - 1] > c))) {
                cl[j] = cl[j - 1];
                score[j] = score[j - 1];
                --j;
            }
            cl[j] = c;
            score[j] = s;
        }
        free(score);
    }
}

/* ---------------------------------------------------------------- search */

typedef struct {
    /* reference-format index (global point order) */
    uint32_t n, d8, a, ncells, degree, cross_e;
    const uint16_t* vec16;   /* n x d8 fp16 bits, alpha-scaled (orc_f2h) */
    const float* attrs;      /* n x a */
    const uint32_t* cell_of; /* n: grid cell of each point (global_pid) */
    const uint32_t* graphs;  /* concatenated per-cell graphs, cell order, local ids */
    const uint32_t* cross;   /* n x (ncells * cross_e) local ids in the target cell */
    /* byte-row codec (codec != 0): rows of d16 bytes, per-element scale and bias */
    uint32_t codec;          /* 0 = fp16 rows (vec16), 1 = int8, 2 = uint8 (vec8) */
    uint32_t d16;
    const uint8_t* vec8;     /* n x d16 */
    const float* scale;      /* d16 (0 past dim) */
    const float* bias;       /* d16: zero_point + 128 (int8) or zero_point (uint8) */
} orc_index;

typedef struct {
    uint32_t L, K, width, max_iter, postfilter;
    float prefilter;
    uint32_t n_entry; /* number of entry points (= degree in the reference) */
} orc_params;

typedef struct {
    float d;
    uint32_t w; /* position | flags */
} ent;

static inline int ent_less(ent x, ent y) {
    uint32_t a = x.w == ORC_EMPTY ? ORC_EMPTY : (x.w & ORC_POSMASK);
    uint32_t b = y.w == ORC_EMPTY ? ORC_EMPTY : (y.w & ORC_POSMASK);
    return x.d < y.d || (x.d == y.d && a < b);
}

static void ent_sort(ent* v, uint32_t n) {
    for (uint32_t i = 1; i < n; ++i) {
        ent x = v[i];
        uint32_t j = i;
        while (j > 0 && ent_less(x, v[j - 1])) {
            v[j] = v[j - 1];
            --j;
        }
        v[j] = x;
    }
}

/*
 * Merge the sorted batch b[0..nb) into the sorted list t[0..cap) (merge_top,
 * gpu_graph.cu:162-222).  When rl != NULL, list items pushed out that carry the
 * in-range flag are offered to the recycle list rl[0..rlcap) (merge_top_with_recycle_list,
 * gpu_graph.cu:482-581, followed by merge_top into the recycle list, :3419-3425).
 */
static void merge_into(ent* t, uint32_t cap, const ent* b, uint32_t nb, ent* rl, uint32_t rlcap, ent* tmp) {
    uint32_t i = 0, j = 0, o = 0;
    uint32_t total = cap + nb;
    ent* ev = tmp + cap; /* evicted list items, in order */
    uint32_t nev = 0;
    for (uint32_t r = 0; r < total; ++r) {
        ent x;
        int from_t;
        if (j >= nb || (i < cap && !ent_less(b[j], t[i]))) {
            x = t[i++];
            from_t = 1;
        } else {
            x = b[j++];
            from_t = 0;
        }
        if (o < cap)
            tmp[o++] = x;
        else if (from_t && x.w != ORC_EMPTY && (x.w & ORC_INRANGE))
            ev[nev++] = x;
    }
    memcpy(t, tmp, sizeof(ent) * cap);
    if (rl && nev) {
        ent* r2 = (ent*)malloc(sizeof(ent) * (rlcap + nev));
        uint32_t a = 0, c = 0, k = 0;
        while (k < rlcap) {
            if (c >= nev || (a < rlcap && !ent_less(ev[c], rl[a])))
                r2[k++] = rl[a++];
            else
                r2[k++] = ev[c++];
        }
        memcpy(rl, r2, sizeof(ent) * rlcap);
        free(r2);
    }
}

typedef struct {
    const orc_index* ix;
    const uint32_t* seg;   /* ncells + 1 */
    const uint32_t* g_of;  /* position -> global id */
    const uint32_t* p_of;  /* global id -> position */
    const uint16_t* q16;   /* d8 */
    const float* qv;       /* d16: fp32 query * f2h_factor, zero padded (byte codecs) */
    const float* lb;
    const float* rb;
    uint64_t* stats; /* n_dist, n_exp, n_cross, n_hops */
} qctx;

static inline float row_dist(const qctx* c, uint32_t g) {
    const orc_index* ix = c->ix;
    if (ix->codec == 0) return orc_dist16(c->q16, ix->vec16 + (size_t)g * ix->d8, ix->d8);
    return orc_dist8(c->qv, ix->vec8 + (size_t)g * ix->d16, ix->scale, ix->bias, ix->codec == 1 ? 0x80u : 0u,
                     ix->d16);
}

static inline ent evaluate(const qctx* c, uint32_t pos) {
    uint32_t g = c->g_of[pos];
    ent e;
    e.d = row_dist(c, g);
    e.w = pos | (in_box(c->ix->attrs + (size_t)g * c->ix->a, c->lb, c->rb, c->ix->a) ? ORC_INRANGE : 0);
    c->stats[0]++;
    return e;
}

/*
 * One query of gpu_graph.cu:3270-4131.
 *
 * Graph route (taken when the query has fewer than `postfilter` cells and its global
 * box count is above `prefilter`, :3377):
 *   list T (L entries) and recycle list RL (K entries) start empty (:3330-3357);
 *   the entry set of the first cell is the n_entry entry local ids (:3349);
 *   for each cell in order:
 *     (a) evaluate the entry set, sort it, merge into T; in-range items pushed out of T
 *         go to RL (:3385-3425);
 *     (b) repeat until T has no unexplored entry or max_iter rounds: take the first
 *         `width` unexplored entries of T (width = 1 in the reference, :3457-3495), mark
 *         them explored, evaluate their not-yet-seen neighbours in this cell's graph,
 *         sort, merge into T with recycling (:3500-3546);
 *     (c) mark all of T explored (:3555);
 *     (d) if another cell follows: the first min(L,64) non-empty entries of T each give
 *         their cross_e cross edges into the next cell (:3564-3590); the distinct
 *         targets plus, to make up cross_e slots per entry, the smallest local ids of
 *         the next cell not among them (the reference's fallback scan, :3582-3588) are
 *         evaluated and sorted; the first n_entry become the next entry set, the
 *         following 64 are merged into T WITHOUT recycling (:3634-3635), the rest are
 *         dropped.
 *   Finally the in-range entries of T and RL give the K results (:4025-4048).
 *
 * "Not yet seen": a point evaluated in (a), (b) or kept in (d) is not evaluated again
 * in this cell.  The reference's forgetful 2048-slot hash (:3441-3454) may evaluate
 * such a point again; the CUDA port's hash may too.  Both are harmless: a point not in
 * T was compared against T already and lost, T's worst entry only improves, so the
 * repeat loses again and is not recycled.  Points dropped in (d) are not marked.
 *
 * Exact route (:3788-4022): every in-range point of the query's cells competes, K best
 * by (distance, position).  Taken when the box count / n <= prefilter, or when the
 * query has >= postfilter cells (the reference then returns an empty list, :3377 +
 * :4025; the scan is what the route is for).
 */
static int route_exact(const orc_index* ix, const orc_params* p, uint32_t nc, uint32_t box_count) {
    float prop = (float)((double)box_count / (double)ix->n); /* real_dataset_adapter.cuh:380 */
    return (nc >= p->postfilter) || (prop <= p->prefilter);
}

/* cl[0..nc) are the cells to visit; `exact` the route (route_exact of the query's full
 * cell list).  Results: K (global id, distance) pairs, ORC_EMPTY / +inf padded. */
static void search_one(const qctx* c, const orc_params* p, const uint32_t* cl, uint32_t nc, int exact,
                       const uint32_t* entry, uint32_t* out_ids, float* out_d) {
    const orc_index* ix = c->ix;
    const uint32_t K = p->K, L = p->L, R = ix->degree;
    for (uint32_t k = 0; k < K; ++k) {
        out_ids[k] = ORC_EMPTY;
        out_d[k] = INFINITY;
    }
    if (nc == 0) return;
    if (exact) {
        orc_pair* best = (orc_pair*)malloc(sizeof(orc_pair) * K);
        uint32_t nb = 0;
        for (uint32_t ci = 0; ci < nc; ++ci) {
            uint32_t cell = cl[ci];
            for (uint32_t pos = c->seg[cell]; pos < c->seg[cell + 1]; ++pos) {
                uint32_t g = c->g_of[pos];
                if (!in_box(ix->attrs + (size_t)g * ix->a, c->lb, c->rb, ix->a)) continue;
                c->stats[0]++;
                orc_pair v = {row_dist(c, g), pos};
                topk_insert(best, &nb, K, v);
            }
        }
        for (uint32_t k = 0; k < nb; ++k) {
            out_ids[k] = c->g_of[best[k].id];
            out_d[k] = best[k].d;
        }
        free(best);
        return;
    }
    const uint32_t width = p->width ? p->width : 1;
    const uint32_t hop_n = L < 64 ? L : 64;
    const uint32_t E = ix->cross_e;
    uint32_t bcap = width * R;
    if (bcap < p->n_entry) bcap = p->n_entry;
    if (bcap < hop_n * E) bcap = hop_n * E;
    ent* T = (ent*)malloc(sizeof(ent) * L);
    ent* RL = (ent*)malloc(sizeof(ent) * K);
    ent* B = (ent*)malloc(sizeof(ent) * bcap);
    ent* tmp = (ent*)malloc(sizeof(ent) * (L + bcap));
    uint8_t* seen = (uint8_t*)calloc(ix->n, 1);
    uint32_t* touched = (uint32_t*)malloc(sizeof(uint32_t) * 64);
    uint32_t ntouched = 0, touched_cap = 64;
#define MARK(pos)                                                                                  \
    do {                                                                                           \
        seen[pos] = 1;                                                                             \
        if (ntouched == touched_cap) {                                                             \
            touched_cap *= 2;                                                                      \
            touched = (uint32_t*)realloc(touched, sizeof(uint32_t) * touched_cap);                 \
        }                                                                                          \
        touched[ntouched++] = pos;                                                                 \
    } while (0)
    for (uint32_t i = 0; i < L; ++i) T[i] = (ent){INFINITY, ORC_EMPTY};
    for (uint32_t i = 0; i < K; ++i) RL[i] = (ent){INFINITY, ORC_EMPTY};
    /* entry set of the first cell */
    uint32_t nbt = 0;
    {
        uint32_t cell = cl[0], sz = c->seg[cell + 1] - c->seg[cell];
        for (uint32_t i = 0; i < p->n_entry; ++i) {
            if (entry[i] >= sz) continue;
            uint32_t pos = c->seg[cell] + entry[i];
            if (seen[pos]) continue;
            MARK(pos);
            B[nbt++] = evaluate(c, pos);
        }
    }
    for (uint32_t ci = 0; ci < nc; ++ci) {
        uint32_t cell = cl[ci];
        /* (a) */
        ent_sort(B, nbt);
        merge_into(T, L, B, nbt, RL, K, tmp);
        /* (b) */
        for (uint32_t it = 0; it < p->max_iter; ++it) {
            uint32_t picked[64], np = 0;
            for (uint32_t i = 0; i < L && np < width; ++i)
                if (T[i].w != ORC_EMPTY && !(T[i].w & ORC_EXPLORED)) {
                    T[i].w |= ORC_EXPLORED;
                    picked[np++] = T[i].w & ORC_POSMASK;
                }
            if (np == 0) break;
            c->stats[1] += np;
            nbt = 0;
            for (uint32_t k = 0; k < np; ++k) {
                const uint32_t* nbrs = ix->graphs + (size_t)picked[k] * R; /* rows in position order */
                for (uint32_t j = 0; j < R; ++j) {
                    uint32_t loc = nbrs[j];
                    if (loc >= c->seg[cell + 1] - c->seg[cell]) continue;
                    uint32_t pos = c->seg[cell] + loc;
                    if (seen[pos]) continue;
                    MARK(pos);
                    B[nbt++] = evaluate(c, pos);
                }
            }
            ent_sort(B, nbt);
            merge_into(T, L, B, nbt, RL, K, tmp);
        }
        /* (c) */
        for (uint32_t i = 0; i < L; ++i)
            if (T[i].w != ORC_EMPTY) T[i].w |= ORC_EXPLORED;
        /* (d) */
        nbt = 0;
        if (ci + 1 < nc) {
            uint32_t next = cl[ci + 1], base = c->seg[next], sz = c->seg[next + 1] - base;
            uint32_t V = 0;
            for (uint32_t i = 0; i < hop_n; ++i)
                if (T[i].w != ORC_EMPTY) {
                    uint32_t g = c->g_of[T[i].w & ORC_POSMASK];
                    ++V;
                    c->stats[2]++;
                    for (uint32_t j = 0; j < E; ++j) {
                        uint32_t loc = ix->cross[(size_t)g * ix->ncells * E + (size_t)next * E + j];
                        if (loc >= sz) continue;
                        uint32_t pos = base + loc;
                        int dup = 0;
                        for (uint32_t k = 0; k < nbt && !dup; ++k) dup = (B[k].w & ORC_POSMASK) == pos;
                        if (!dup) B[nbt++] = (ent){0.0f, pos};
                    }
                }
            uint32_t want = V * E;
            uint32_t ndist = nbt;
            for (uint32_t loc = 0; loc < sz && nbt < want; ++loc) {
                uint32_t pos = base + loc;
                int dup = 0;
                for (uint32_t k = 0; k < ndist && !dup; ++k) dup = (B[k].w & ORC_POSMASK) == pos;
                if (!dup) B[nbt++] = (ent){0.0f, pos};
            }
            for (uint32_t k = 0; k < nbt; ++k) B[k] = evaluate(c, B[k].w);
            ent_sort(B, nbt);
            c->stats[3]++;
            uint32_t ne = nbt < p->n_entry ? nbt : p->n_entry;
            uint32_t nm = nbt - ne < 64 ? nbt - ne : 64;
            /* new cell: forget the previous cell's marks (its points never come back) */
            for (uint32_t k = 0; k < ntouched; ++k) seen[touched[k]] = 0;
            ntouched = 0;
            for (uint32_t k = 0; k < ne + nm; ++k) MARK(B[k].w & ORC_POSMASK);
            merge_into(T, L, B + ne, nm, NULL, 0, tmp);
            nbt = ne; /* B[0..ne) is the next entry set, already evaluated */
        }
    }
    /* final post-filter + recycle merge */
    uint32_t o = 0;
    ent* fin = (ent*)malloc(sizeof(ent) * (L + K));
    for (uint32_t i = 0; i < L; ++i)
        if (T[i].w != ORC_EMPTY && (T[i].w & ORC_INRANGE)) fin[o++] = T[i];
    for (uint32_t i = 0; i < K; ++i)
        if (RL[i].w != ORC_EMPTY) fin[o++] = RL[i];
    ent_sort(fin, o);
    for (uint32_t k = 0; k < K && k < o; ++k) {
        out_ids[k] = c->g_of[fin[k].w & ORC_POSMASK];
        out_d[k] = fin[k].d;
    }
#undef MARK
    free(fin);
    free(T);
    free(RL);
    free(B);
    free(tmp);
    free(seen);
    free(touched);
}

/* Forward declaration (defined below). */
static void make_positions(const orc_index* ix, uint32_t** seg_out, uint32_t** g_out, uint32_t** p_out);

/*
 * full_graph_search.cuh:984-997 (assemble_edges): one row per point, `reserve` neighbours
 * per cell -- in the point's own cell the first `reserve` entries of its cell-graph row,
 * in every other cell its first `reserve` cross edges -- slot j*reserve + e for cell j.
 * Rows and entries are positions (the reference writes global ids, rows by global id);
 * an entry that is not a point of its cell is ORC_EMPTY.  out: n x (ncells*reserve).
 */
void orc_assemble(const orc_index* ix, uint32_t reserve, uint32_t* out) {
    uint32_t *seg, *g_of, *p_of;
    make_positions(ix, &seg, &g_of, &p_of);
    const uint32_t P = ix->ncells, R = ix->degree, E = ix->cross_e, D = P * reserve;
    for (uint32_t pos = 0; pos < ix->n; ++pos) {
        const uint32_t g = g_of[pos], own = ix->cell_of[g];
        for (uint32_t j = 0; j < P; ++j) {
            const uint32_t base = seg[j], sz = seg[j + 1] - seg[j];
            for (uint32_t e = 0; e < reserve; ++e) {
                uint32_t loc = ORC_EMPTY;
                if (j == own)
                    loc = e < R ? ix->graphs[(size_t)pos * R + e] : ORC_EMPTY;
                else
                    loc = e < E ? ix->cross[(size_t)g * P * E + (size_t)j * E + e] : ORC_EMPTY;
                out[(size_t)pos * D + (size_t)j * reserve + e] = loc < sz ? base + loc : ORC_EMPTY;
            }
        }
    }
    free(seg);
    free(g_of);
    free(p_of);
}

/*
 * full_graph_search.cuh:179-593 (full_graph_search_postfiltering): beam search over the
 * assembled graph `fg` (orc_assemble, `deg` entries per row) of the whole index, filtered
 * by the box only at the end.  The entry set is entry_pos[0..n_entry) (positions); list T
 * of L entries; each round expands the first `width` unexplored entries of T (width 1 in the
 * reference, :394-418), evaluates their not-yet-seen neighbours, sorts and merges them into
 * T (:421-511, no recycle list); the search stops when T has no unexplored entry or after
 * max_iter rounds.  The in-range entries of T in list order give the K results (:579-592).
 */
void orc_search_fullgraph(const orc_index* ix, const orc_params* p, const uint32_t* fg, uint32_t deg,
                          const float* queries, uint32_t dim, float alpha, const float* lb, const float* rb,
                          uint32_t qnum, const uint32_t* entry_pos, uint32_t* ids_out, float* dist_out,
                          uint64_t* stats, int threads) {
    uint32_t *seg, *g_of, *p_of;
    make_positions(ix, &seg, &g_of, &p_of);
    uint64_t tot[4] = {0, 0, 0, 0};
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#endif
#pragma omp parallel
    {
        uint64_t st[4] = {0, 0, 0, 0};
        const uint32_t L = p->L, K = p->K, width = p->width ? p->width : 1;
        uint32_t bcap = width * deg > p->n_entry ? width * deg : p->n_entry;
        uint16_t* q16 = (uint16_t*)malloc(sizeof(uint16_t) * ix->d8);
        float* qv = (float*)calloc(ix->d16 > dim ? ix->d16 : dim, sizeof(float));
        ent* T = (ent*)malloc(sizeof(ent) * L);
        ent* B = (ent*)malloc(sizeof(ent) * bcap);
        ent* tmp = (ent*)malloc(sizeof(ent) * (L + bcap));
        uint8_t* seen = (uint8_t*)calloc(ix->n ? ix->n : 1, 1);
        uint32_t* touched = (uint32_t*)malloc(sizeof(uint32_t) * (L + bcap) * 64);
#pragma omp for schedule(dynamic, 1)
        for (long q = 0; q < (long)qnum; ++q) {
            orc_f2h(queries + (size_t)q * dim, 1, dim, ix->d8, alpha, q16);
            for (uint32_t i = 0; i < dim; ++i) qv[i] = queries[(size_t)q * dim + i] * alpha;
            qctx c = {ix, seg, g_of, p_of, q16, qv, lb + q * ix->a, rb + q * ix->a, st};
            uint32_t nt = 0, nbt = 0;
            for (uint32_t i = 0; i < L; ++i) T[i] = (ent){INFINITY, ORC_EMPTY};
            for (uint32_t i = 0; i < p->n_entry; ++i) {
                const uint32_t pos = entry_pos[i];
                if (pos >= ix->n || seen[pos]) continue;
                seen[pos] = 1;
                touched[nt++] = pos;
                B[nbt++] = evaluate(&c, pos);
            }
            ent_sort(B, nbt);
            merge_into(T, L, B, nbt, NULL, 0, tmp);
            for (uint32_t it = 0; it < p->max_iter; ++it) {
                uint32_t picked[64], np = 0;
                for (uint32_t i = 0; i < L && np < width; ++i)
                    if (T[i].w != ORC_EMPTY && !(T[i].w & ORC_EXPLORED)) {
                        T[i].w |= ORC_EXPLORED;
                        picked[np++] = T[i].w & ORC_POSMASK;
                    }
                if (np == 0) break;
                st[1] += np;
                nbt = 0;
                for (uint32_t k = 0; k < np; ++k)
                    for (uint32_t j = 0; j < deg; ++j) {
                        const uint32_t pos = fg[(size_t)picked[k] * deg + j];
                        if (pos == ORC_EMPTY || seen[pos]) continue;
                        seen[pos] = 1;
                        if (nt < (L + bcap) * 64) touched[nt++] = pos;
                        B[nbt++] = evaluate(&c, pos);
                    }
                ent_sort(B, nbt);
                merge_into(T, L, B, nbt, NULL, 0, tmp);
            }
            uint32_t o = 0;
            for (uint32_t i = 0; i < L && o < K; ++i)
                if (T[i].w != ORC_EMPTY && (T[i].w & ORC_INRANGE)) {
                    ids_out[(size_t)q * K + o] = g_of[T[i].w & ORC_POSMASK];
                    dist_out[(size_t)q * K + o] = T[i].d;
                    ++o;
                }
            for (; o < K; ++o) {
                ids_out[(size_t)q * K + o] = ORC_EMPTY;
                dist_out[(size_t)q * K + o] = INFINITY;
            }
            if (nt < (L + bcap) * 64) {
                for (uint32_t k = 0; k < nt; ++k) seen[touched[k]] = 0;
            } else {
                memset(seen, 0, ix->n);
            }
        }
#pragma omp critical
        for (int i = 0; i < 4; ++i) tot[i] += st[i];
        free(q16);
        free(qv);
        free(T);
        free(B);
        free(tmp);
        free(seen);
        free(touched);
    }
    if (stats)
        for (int i = 0; i < 4; ++i) stats[i] += tot[i];
    free(seg);
    free(g_of);
    free(p_of);
}

/* Cell-major positions (tools.cuh:862-889 get_idx_mapper): seg[c] .. seg[c+1]-1 are the
 * points of cell c in increasing global id; g_of maps position -> id, p_of id -> position. */
static void make_positions(const orc_index* ix, uint32_t** seg_out, uint32_t** g_out, uint32_t** p_out) {
    uint32_t* seg = (uint32_t*)calloc(ix->ncells + 1, sizeof(uint32_t));
    uint32_t* g_of = (uint32_t*)malloc(sizeof(uint32_t) * (ix->n ? ix->n : 1));
    uint32_t* p_of = (uint32_t*)malloc(sizeof(uint32_t) * (ix->n ? ix->n : 1));
    for (uint32_t i = 0; i < ix->n; ++i) seg[ix->cell_of[i] + 1]++;
    for (uint32_t c = 0; c < ix->ncells; ++c) seg[c + 1] += seg[c];
    uint32_t* fill = (uint32_t*)calloc(ix->ncells ? ix->ncells : 1, sizeof(uint32_t));
    for (uint32_t i = 0; i < ix->n; ++i) {
        uint32_t c = ix->cell_of[i];
        uint32_t pos = seg[c] + fill[c]++;
        g_of[pos] = i;
        p_of[i] = pos;
    }
    free(fill);
    *seg_out = seg;
    *g_out = g_of;
    *p_out = p_of;
}

/*
 * Batch driver (gpu_graph.cu:12464-12616 minus the launch): cells/counts/offsets are the
 * ordered CSR from orc_plan_cells + orc_order_cells; box_counts from orc_count_in_box
 * (only read when prefilter > 0); entry[] the entry local ids.  Graph rows in
 * ix->graphs are stored per cell in local order, i.e. row index = position.
 * stats (may be NULL) accumulates n_dist, n_exp, n_cross, n_hops.
 */
void orc_search(const orc_index* ix, const orc_params* p, const float* queries, uint32_t dim, float alpha,
                const float* lb, const float* rb, uint32_t qnum, const uint32_t* counts, const uint32_t* offsets,
                const uint32_t* cells, const uint32_t* box_counts, const uint32_t* entry, uint32_t* ids_out,
                float* dist_out, uint64_t* stats, int threads) {
    uint32_t *seg, *g_of, *p_of;
    make_positions(ix, &seg, &g_of, &p_of);
    uint64_t tot[4] = {0, 0, 0, 0};
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#endif
#pragma omp parallel
    {
        uint64_t st[4] = {0, 0, 0, 0};
        uint16_t* q16 = (uint16_t*)malloc(sizeof(uint16_t) * ix->d8);
        float* qv = (float*)calloc(ix->d16 > dim ? ix->d16 : dim, sizeof(float));
#pragma omp for schedule(dynamic, 1)
        for (long q = 0; q < (long)qnum; ++q) {
            orc_f2h(queries + (size_t)q * dim, 1, dim, ix->d8, alpha, q16);
            for (uint32_t i = 0; i < dim; ++i) qv[i] = queries[(size_t)q * dim + i] * alpha;
            qctx c = {ix, seg, g_of, p_of, q16, qv, lb + q * ix->a, rb + q * ix->a, st};
            int exact = route_exact(ix, p, counts[q], box_counts ? box_counts[q] : ix->n);
            search_one(&c, p, cells + offsets[q], counts[q], exact, entry, ids_out + (size_t)q * p->K,
                       dist_out + (size_t)q * p->K);
        }
#pragma omp critical
        for (int i = 0; i < 4; ++i) tot[i] += st[i];
        free(q16);
        free(qv);
    }
    if (stats)
        for (int i = 0; i < 4; ++i) stats[i] += tot[i];
    free(seg);
    free(g_of);
    free(p_of);
}

/*
 * Search over batches of cells (the out-of-core driver,
 * big_dataset_adapterV3.cuh:3321-3715, with its per-batch kernel :754-1390 and the
 * per-batch cell lists of fill_partition_info03, tools.cuh:1646-1670).
 * batch_of[c] is the batch holding cell c, or ORC_EMPTY when c is searched in no batch.
 * For batch b = 0 .. n_batches-1 each query visits the cells of its planned list that
 * batch b holds, in planned order, with search_one (entry set in the first of them; the
 * route is decided once from the query's full list); the K results of the batch are
 * merged into the query's running K best by (distance, position), which replaces the
 * reference's host-side merge of each batch's list (:3347-3395).
 */
void orc_search_batched(const orc_index* ix, const orc_params* p, const float* queries, uint32_t dim, float alpha,
                        const float* lb, const float* rb, uint32_t qnum, const uint32_t* counts,
                        const uint32_t* offsets, const uint32_t* cells, const uint32_t* box_counts,
                        const uint32_t* entry, const uint32_t* batch_of, uint32_t n_batches, uint32_t* ids_out,
                        float* dist_out, uint64_t* stats, int threads) {
    uint32_t *seg, *g_of, *p_of;
    make_positions(ix, &seg, &g_of, &p_of);
    const uint32_t K = p->K;
    uint64_t tot[4] = {0, 0, 0, 0};
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#endif
#pragma omp parallel
    {
        uint64_t st[4] = {0, 0, 0, 0};
        uint16_t* q16 = (uint16_t*)malloc(sizeof(uint16_t) * ix->d8);
        float* qv = (float*)calloc(ix->d16 > dim ? ix->d16 : dim, sizeof(float));
        uint32_t* sub = (uint32_t*)malloc(sizeof(uint32_t) * (ix->ncells ? ix->ncells : 1));
        uint32_t* bid = (uint32_t*)malloc(sizeof(uint32_t) * K);
        float* bd = (float*)malloc(sizeof(float) * K);
        ent* run = (ent*)malloc(sizeof(ent) * K);
        ent* got = (ent*)malloc(sizeof(ent) * K);
        ent* tmp = (ent*)malloc(sizeof(ent) * 2 * K);
#pragma omp for schedule(dynamic, 1)
        for (long q = 0; q < (long)qnum; ++q) {
            orc_f2h(queries + (size_t)q * dim, 1, dim, ix->d8, alpha, q16);
            for (uint32_t i = 0; i < dim; ++i) qv[i] = queries[(size_t)q * dim + i] * alpha;
            qctx c = {ix, seg, g_of, p_of, q16, qv, lb + q * ix->a, rb + q * ix->a, st};
            const uint32_t* cl = cells + offsets[q];
            int exact = route_exact(ix, p, counts[q], box_counts ? box_counts[q] : ix->n);
            for (uint32_t k = 0; k < K; ++k) run[k] = (ent){INFINITY, ORC_EMPTY};
            for (uint32_t b = 0; b < n_batches; ++b) {
                uint32_t ns = 0;
                for (uint32_t i = 0; i < counts[q]; ++i)
                    if (batch_of[cl[i]] == b) sub[ns++] = cl[i];
                if (ns == 0) continue;
                search_one(&c, p, sub, ns, exact, entry, bid, bd);
                uint32_t ng = 0;
                for (uint32_t k = 0; k < K; ++k)
                    if (bid[k] != ORC_EMPTY) got[ng++] = (ent){bd[k], p_of[bid[k]]};
                merge_into(run, K, got, ng, NULL, 0, tmp);
            }
            for (uint32_t k = 0; k < K; ++k) {
                ids_out[(size_t)q * K + k] = run[k].w == ORC_EMPTY ? ORC_EMPTY : g_of[run[k].w & ORC_POSMASK];
                dist_out[(size_t)q * K + k] = run[k].w == ORC_EMPTY ? INFINITY : run[k].d;
            }
        }
#pragma omp critical
        for (int i = 0; i < 4; ++i) tot[i] += st[i];
        free(q16);
        free(qv);
        free(sub);
        free(bid);
        free(bd);
        free(run);
        free(got);
        free(tmp);
    }
    if (stats)
        for (int i = 0; i < 4; ++i) stats[i] += tot[i];
    free(seg);
    free(g_of);
    free(p_of);
}

/*
 * tools.cuh:456-544: mean over queries of |res ∩ gt| / |gt|, |gt| = 0 counting as 1.
 * ORC_EMPTY entries are not ids and are ignored on both sides.
 */
double orc_recall(const uint32_t* res, uint32_t kr, const uint32_t* gt, uint32_t kg, uint32_t qnum) {
    double total = 0.0;
    for (uint32_t q = 0; q < qnum; ++q) {
        uint32_t ng = 0, hit = 0;
        for (uint32_t j = 0; j < kg; ++j) {
            uint32_t g = gt[(size_t)q * kg + j];
            if (g == ORC_EMPTY) continue;
            ++ng;
            for (uint32_t i = 0; i < kr; ++i)
                if (res[(size_t)q * kr + i] == g) {
                    ++hit;
                    break;
                }
        }
        total += ng ? (double)hit / ng : 1.0;
    }
    return qnum ? total / qnum : 1.0;
}
