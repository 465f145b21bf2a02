/*
 * garfield.h -- C ABI of garfield_b200, a B200 (sm_100a) implementation of the
 * Garfield GMG query path: range-filtered approximate nearest-neighbour search over a
 * grid of per-cell graphs joined by cross-cell edges.
 *
 * The reference (ZJU-DAILY/Garfield) has no library surface; its query path is a set
 * of templated host functions inside one CUDA translation unit.  Each entry point
 * below names the reference function it replaces.  Conventions:
 *   - every call returns gf_status (GF_OK = 0); nothing exits or prints;
 *     gf_last_error() holds a message for the calling thread;
 *   - pointers documented "device" are CUDA device pointers on the index's device,
 *     "host" are ordinary host pointers; sizes are element counts;
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream);
 *     calls only enqueue work unless they return host data;
 *   - ids returned to callers are the reference's global point ids (row numbers of
 *     the data file); 0xFFFFFFFF marks "no result".
 */
#ifndef GARFIELD_B200_H
#define GARFIELD_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    GF_OK = 0,
    GF_ERR_ARG = 1,     /* invalid argument or size */
    GF_ERR_IO = 2,      /* file cannot be opened / read / written */
    GF_ERR_FORMAT = 3,  /* file or array contents inconsistent */
    GF_ERR_OOM = 4,     /* device or host allocation failed */
    GF_ERR_CUDA = 5,    /* CUDA runtime error */
    GF_ERR_TIMEOUT = 6, /* a bounded wait ran out */
    GF_ERR_STATE = 7    /* call out of order (e.g. search before plan) */
} gf_status;

#define GF_NO_ID 0xFFFFFFFFu

typedef struct gf_index gf_index;
typedef struct gf_plan gf_plan;

/*
 * Host description of an index in the reference's on-disk layout (global point order).
 * Replaces the loading block of real_dataset_test_multiD (realdataset_search.cu:2118-2393):
 * get_graph_info (check.cu:406), load_grid_infos/load2GPU (real_dataset_adapter.cuh:563,589),
 * get_idx_mapper (tools.cuh:862), load_result for the global graph (tools.cuh:205),
 * load_attrs (tools.cuh:747), f2h (tools.cuh:308), load_clustering (tools.cuh:569).
 */
typedef struct {
    uint32_t n;            /* points */
    uint32_t dim;          /* vector dimension */
    uint32_t n_attr;       /* attributes per point (grid dimensions) */
    const float* vectors;  /* host, n x dim fp32 */
    const float* attrs;    /* host, n x n_attr (integer attributes converted to float) */
    const uint32_t* grid;  /* host, n_attr slice counts */
    const float* l_quant;  /* host, sum(grid): closed lower bound of each slice, per dim */
    const float* r_quant;  /* host, sum(grid): closed upper bound of each slice */
    const uint32_t* cell_of; /* host, n: grid cell of each point (grid_info global_pid) */
    uint32_t degree;       /* per-cell graph degree R */
    const uint32_t* graphs; /* host, n x degree: per-cell graphs concatenated in cell order,
                               rows in local order, entries = local ids in the same cell */
    uint32_t cross_e;      /* cross-cell edges per (point, cell) E */
    const uint32_t* cross; /* host, n x (ncells*cross_e), global row order, local ids */
    uint32_t n_clusters;   /* 0 = no cluster-guided ordering (cells keep id order) */
    const int32_t* labels; /* host, n cluster labels (cluster.bin), or NULL */
    float f2h_factor;      /* --f2h_factor: vectors are stored as half(x * f2h_factor) */
    uint32_t keep_fp32;    /* 1 = also keep fp32 vectors on the device (gf_bruteforce) */
    uint32_t host_graph;   /* 1 = keep the graphs and cross edges in pinned host memory and
                              copy them to the device per batch of cells (gf_search_batched;
                              the dataset-resident out-of-core mode of
                              big_dataset_adapterV3.cuh:3321) */
    const uint32_t* shard_cells; /* host, or NULL: build a shard holding only these cells'
                              vectors, graph rows and the cross edges among them (cell
                              sharding over GPUs).  Positions, attributes, ids, the planner
                              data and the entry sequence stay those of the whole index, so
                              shard results merge by (distance, position) (gf_search_keys,
                              gf_merge_keys).  Not with host_graph or keep_fp32. */
    uint32_t n_shard_cells;
    /* Stored row format.  0 = fp16 (half(x * f2h_factor)); 1 = int8 per-dimension affine
     * (the out-of-core codec, production_adapter.cuh:286-383): codes = NULL quantises
     * vectors * f2h_factor here (gf_quantize_i8_host), else codes / code_scales /
     * code_zero_points are the quantised rows (n x dim, global order) and their parameters,
     * e.g. from a .q file; 2 = uint8 rows (u8bin data, big_dataset_adapterV3.cuh:2802-2810)
     * in codes, decoded scale * (q - zero_point), default scale 0.01 and zero point 0.
     * Byte rows are compared with the fp32 query * f2h_factor (gf_search, orc_dist8). */
    uint32_t codec;
    const uint8_t* codes;
    const float* code_scales;
    const int32_t* code_zero_points;
    /* 1 = store the cross-cell edges of spokesmen only (the "extreme" compression of
     * compress_global_graph_extreme, tools.cuh:917-1010; see gf_spokesman_host): a point's
     * hop into another cell uses its spokesman's edges.  Not with host_graph or shard_cells. */
    uint32_t cross_spokesman;
} gf_index_desc;

/* Paths of the reference's index files (realdataset_search flags, README.md:101-170). */
typedef struct {
    const char* data_path;    /* --data_path  .fvecs */
    const char* cagra_prefix; /* --cagra_prefix  graph of cell c = prefix + c + suffix */
    const char* cagra_suffix; /* --cagra_suffix */
    const char* global_graph; /* --global_graph  cross-cell edges */
    const char* grid;         /* --grid  grid_info */
    const char* attrs;        /* --attrs  attrs.bin */
    const char* cluster;      /* --cluster  cluster.bin, or NULL */
    uint32_t degree;          /* --degree */
    float f2h_factor;         /* --f2h_factor */
    uint32_t keep_fp32;
    uint32_t host_graph;      /* as gf_index_desc.host_graph */
    uint32_t codec;           /* as gf_index_desc.codec; 2 reads data_path as u8bin */
    const char* quantized;    /* codec 1: .q file with the codes (NULL: quantise the data) */
    /* Uniform grid (normaldataset_search, normaldataset_search.cu:1748-2104), used when
     * grid is NULL: attribute j is cut into uniform_shape[j] equal slices of
     * [uniform_lo, uniform_hi) (the reference compiles shape {16} and [0, 1e6) in);
     * slice s holds integer values lo + s*w .. lo + (s+1)*w - 1, w = (hi - lo) / shape. */
    uint32_t uniform_dims;
    const uint32_t* uniform_shape;
    float uniform_lo, uniform_hi;
} gf_index_files;

/* Search knobs.  The defaults (gf_search_defaults) are the reference's values. */
typedef struct {
    uint32_t L;          /* candidate list length ("ef", realdataset_search.cu:2757) */
    uint32_t k;          /* results per query (10 in the reference, :2495) */
    uint32_t width;      /* list entries expanded per round (1 in the reference) */
    uint32_t max_iter;   /* rounds per cell (MAX_ITER = 10000, gpu_graph.cu:39) */
    uint32_t n_entry;    /* entry points of the first cell (= degree in the reference) */
    uint32_t postfilter; /* --postfilter: queries with >= this many cells scan exactly */
    uint32_t hash_slots; /* visited-hash slots per query, power of two; 0 = automatic */
    uint32_t test_wait;  /* 0 in normal use.  Test hook for the timeout path: a row-staging
                            wait gives up after test_wait polls, and every staging batch
                            expects 16 bytes more than it copies, so no wait completes; the
                            warps stop, gf_search_stats.n_timeouts counts them and
                            gf_search_host returns GF_ERR_TIMEOUT. */
    uint32_t exact_tc;   /* 0 = the reference's exact route (fp16 distances over the in-box points
                            of the query's cells, gpu_graph.cu:3788-4022).  1 = queries that take
                            the exact route (postfilter, plan prefilter) are answered by the
                            tensor-core exact scan of gf_bruteforce instead: canonical fp32
                            distances of the fp32 rows, ids ordered by (distance, global id).
                            Needs keep_fp32, dim <= 1024 and k <= 128; gf_search and
                            gf_search_host only (GF_ERR_ARG for batched, sharded, full-graph and
                            no-allocation searches). */
    uint32_t route;      /* 0 = the reference's routing (postfilter, plan prefilter).  1 = also
                            by cost (no counterpart in the reference, which has only the two
                            thresholds): a query with nc planned cells and b in-box points goes
                            to the tensor-core exact scan when b < GF_ROUTE_ROWS_PER_SLOT * nc *
                            (L + 64), an estimate that the scan of its in-box rows costs less
                            than walking L list slots (plus a hop's 64) in each of its cells.
                            Needs exact_tc = 1.  b is the plan's exact box count when the plan
                            was built with prefilter > 0, else an estimate the search makes from
                            the index's attribute tiles (the points of tiles inside the box plus
                            half of those of tiles that meet it in part). */
} gf_search_params;

/* Tensor-core exact-scan rows that cost about as much as one list slot of one cell of the
 * graph route (gf_search_params.route = 1), from B200 measurements of both routes at
 * 96- and 128-dim rows, k = 10 and 100 (1M points: config 2 at 1% and 10% boxes, the
 * configuration-3 shape at 5% boxes). */
#define GF_ROUTE_ROWS_PER_SLOT 150u

/* Per-search counters (device-side, summed over queries). */
typedef struct {
    uint64_t n_dist;    /* distance evaluations */
    uint64_t n_exp;     /* expanded list entries */
    uint64_t n_cross;   /* cross-edge rows read */
    uint64_t n_hops;    /* cell-to-cell hops */
    uint64_t n_exact;   /* queries answered by the exact route */
    uint64_t n_queries;
    uint64_t n_timeouts; /* row-staging waits that ran out (the warp then stopped; any
                            nonzero value makes gf_search_host return GF_ERR_TIMEOUT), plus
                            tensor-core waits of the planner that ran out */
    uint64_t n_plan_fallbacks; /* queries whose 4 nearest centroids the tensor-core planner
                            could not narrow below its candidate cap (exact scan instead) */
    uint64_t n_plan_reranked; /* centroids the tensor-core planner re-ranked with the exact
                            distance (those its error bound could not rule out) */
} gf_search_stats;

typedef struct {
    uint32_t n, dim, n_attr, n_cells, degree, cross_e, n_clusters;
    uint32_t d_stored;       /* stored row length (dim rounded up to 8) */
    uint32_t min_cell_size;  /* entry ids are drawn below this */
    uint32_t cross_rows;     /* points whose cross-cell edges are stored (n, or the spokesmen) */
    uint64_t device_bytes;   /* device memory held by the index */
} gf_index_info;

const char* gf_status_string(gf_status s);
const char* gf_last_error(void);
/* Library version string. */
const char* gf_version(void);

void gf_search_defaults(gf_search_params* p);

/* ---------------------------------------------------------------- index */

/* Build a device index from host arrays.  Replaces the loading block of
 * real_dataset_test_multiD (realdataset_search.cu:2118-2393). */
gf_status gf_index_create(const gf_index_desc* desc, int device, gf_index** out);
/* Load the reference's index files and build a device index (same block, from files). */
gf_status gf_index_open(const gf_index_files* files, int device, gf_index** out);
gf_status gf_index_info_get(const gf_index* idx, gf_index_info* out);
/* Copy the entry local ids (first n of the deterministic entry sequence) to host. */
gf_status gf_index_entry_points(const gf_index* idx, uint32_t n, uint32_t* out_host);
gf_status gf_index_destroy(gf_index* idx);

/* ----------------------------------------------------------------- plan */

/* Plan buffers for up to max_queries queries.  A plan may be destroyed before or after
 * its index; every other call needs the index alive. */
gf_status gf_plan_create(gf_index* idx, uint32_t max_queries, gf_plan** out);
gf_status gf_plan_destroy(gf_plan* plan);

/*
 * Cell intersection + cluster-guided ordering for a batch of queries: the reference's
 * cost1 + cost2.  Replaces intersection_area_mark_little_seg_V2
 * (real_dataset_adapter.cuh:390-519, incl. prefiltering_tag_elements :347) followed by
 * get_partitions_access_order_V2 (gpu_graph.cu:11742-11845).
 *   queries: device, qnum x dim fp32; lb/rb: device, qnum x n_attr closed bounds.
 *   prefilter: --prefilter (box count / n <= prefilter => exact route); the box count
 *   pass runs only when prefilter > 0.
 * On a whole index the centroid stage runs on a stream of the plan, forked from `stream`
 * after the query copy and joined back before the cell ordering with events: all work is
 * ordered on `stream` when the call returns, and the host never waits.
 * On a shard index (gf_index_desc.shard_cells) only the queries with two or more of the
 * shard's cells get their 4 nearest centroids and an ordered cell list: the others keep
 * their cells in increasing id and top4 = 0xFFFFFFFF.  A shard searches only its own cells,
 * so those queries' results there do not depend on the order.
 */
gf_status gf_plan_queries(gf_index* idx, gf_plan* plan, const float* queries, const float* lb, const float* rb,
                          uint32_t qnum, float prefilter, void* stream);

/*
 * Copy the ordered cell lists of the last gf_plan_queries to host (test / inspection).
 * counts, offsets: qnum entries; cells: cap entries; top4: qnum x 4 (may be NULL);
 * box_counts: qnum (may be NULL; valid only when prefilter > 0).  Synchronises.
 */
gf_status gf_plan_read(gf_plan* plan, uint32_t* counts, uint32_t* offsets, uint32_t* cells, uint64_t cap,
                       uint32_t* top4, uint32_t* box_counts);

/*
 * Cell-by-cell filtered beam search of the planned queries.  Replaces
 * batch_graph_search_gpu_with_prefilter_and_postfilter (gpu_graph.cu:12464-12616) and
 * its kernel select_path_contain_attr_filter_V2_without_output_with_post_pre_filter
 * (gpu_graph.cu:3270-4131).  ids_out: device qnum x k global ids; dist_out: device
 * qnum x k squared distances in the stored (scaled) space, or NULL.
 */
gf_status gf_search(gf_index* idx, gf_plan* plan, const gf_search_params* params, uint32_t* ids_out,
                    float* dist_out, void* stream);

/* Counters of the last gf_search on this plan (synchronises the plan's stream). */
gf_status gf_search_stats_read(gf_plan* plan, gf_search_stats* out);

/*
 * End-to-end call from host memory: copies queries and bounds to the device, plans,
 * searches and copies ids (and distances, if dist_host != NULL) back.  Synchronises.
 * The host buffers may be pinned (faster) or pageable.  The device copies live in a
 * buffer owned by the plan, allocated by the first call and grown when a call needs more
 * (qnum x (dim + 2a + 2k) floats); later calls of that size or smaller allocate nothing.
 */
gf_status gf_search_host(gf_index* idx, gf_plan* plan, const gf_search_params* params, const float* queries_host,
                         const float* lb_host, const float* rb_host, uint32_t qnum, float prefilter,
                         uint32_t* ids_host, float* dist_host, void* stream);

/*
 * Search restricted to batches of cells, results merged over the batches.  Replaces the
 * out-of-core driver batch_graph_search_gpu_with_prefilter_batch_process_compressed_graph_
 * T_dataset_resident (big_dataset_adapterV3.cuh:3321-3715) with its per-batch cell lists
 * (fill_partition_info03, tools.cuh:1646) and host-side merge (:3343-3395).
 * batch_cells (host) holds the cells of every batch back to back, batch_sizes[b] (host) how
 * many belong to batch b; a cell may appear in at most one batch, and cells in no batch are
 * not searched.  In batch b every query visits the planned cells that b holds, in planned
 * order, starting from the entry set in the first of them (the route, graph or exact, is
 * decided from the query's full cell list); the batch's k best in-range results are merged
 * into the query's running k best by (distance, position).  One batch holding every cell
 * gives exactly gf_search's results.  For an index with host_graph the graph rows of a
 * batch's cells and the cross-edge blocks between them are copied from pinned host memory
 * on a copy stream, double-buffered, so that the copies of batch b+1 overlap the search of
 * batch b (ordered by stream events).  Needs gf_plan_queries first; ids_out / dist_out
 * (dist may be NULL) device, qnum x k.  Counters (gf_search_stats_read) sum over batches.
 */
gf_status gf_search_batched(gf_index* idx, gf_plan* plan, const gf_search_params* params,
                            const uint32_t* batch_cells, const uint32_t* batch_sizes, uint32_t n_batches,
                            uint32_t* ids_out, float* dist_out, void* stream);

/*
 * Search whose results are merge keys instead of ids: keys_out (device, qnum x k) gets each
 * query's k best as (float bits of the distance << 32) | (position << 2) | flags, sorted
 * ascending, 0xFFFFFFFFFFFFFFFF for "none"; positions are cell-major over the whole index.
 * For a shard index (gf_index_desc.shard_cells) these are the results among the shard's
 * cells; the shards' lists are then exchanged (an all-gather) and merged by gf_merge_keys,
 * the merge step of cell-sharded search over GPUs.  The reference has no multi-GPU path.
 */
gf_status gf_search_keys(gf_index* idx, gf_plan* plan, const gf_search_params* params, uint64_t* keys_out,
                         void* stream);

/*
 * k-way merge of n_lists disjoint sorted key lists per query (device keys laid out
 * [list][query][k], as gathered from gf_search_keys) into the k best ids and distances
 * (device, qnum x k; dist_out may be NULL).  One warp per query ranks every key against
 * the other lists by binary search.
 */
gf_status gf_merge_keys(gf_index* idx, const uint64_t* keys, uint32_t n_lists, uint32_t qnum, uint32_t k,
                        uint32_t* ids_out, float* dist_out, void* stream);

/*
 * Batches of at most max_cells cells for gf_search_batched, grouped so that few queries
 * are split across batches.  The reference uses a fixed random partition of the cells
 * (bigdataset_experiment.cu:271-277); its README (README.md:5) describes minimising the
 * queries active in several batches, which is the objective here: the number of
 * (query, batch) pairs ("splits").  Greedy: a batch starts from the unscheduled cell that
 * most queries visit and adds the cell sharing the most queries with the batch so far.
 * Only cells that some query visits are scheduled.  Outputs (host): batch_cells_out
 * (capacity ncells) and batch_sizes_out (capacity ncells) back to back as
 * gf_search_batched takes them, *n_batches_out, and *splits_out (may be NULL).
 * gf_schedule_batches reads the plan (synchronises its stream); _host takes the plan's
 * cell lists in gf_plan_read's form.
 */
gf_status gf_schedule_batches(gf_plan* plan, uint32_t max_cells, uint32_t* batch_cells_out,
                              uint32_t* batch_sizes_out, uint32_t* n_batches_out, uint64_t* splits_out);
gf_status gf_schedule_batches_host(uint32_t ncells, uint32_t qnum, const uint32_t* counts, const uint32_t* offsets,
                                   const uint32_t* cells, uint32_t max_cells, uint32_t* batch_cells_out,
                                   uint32_t* batch_sizes_out, uint32_t* n_batches_out, uint64_t* splits_out);

/*
 * Full-graph post-filter search, the reference's ablation baseline
 * (full_graph_search_postfiltering over assemble_edges' graph, full_graph_search.cuh:179-997).
 * gf_index_assemble builds the graph on the device: per point `reserve` neighbours per cell
 * (its first `reserve` cell-graph neighbours in its own cell, its first `reserve` cross edges
 * into every other cell; the reference uses reserve = 2) and the entry points (positions,
 * std::mt19937 default seed, draw % n, distinct).  gf_search_fullgraph searches a planned
 * batch (gf_plan_queries) over that graph of the whole index with the same beam rounds as
 * gf_search, without the cell walk or the recycle list, and applies the box to the final
 * list only.  Results as gf_search.
 */
gf_status gf_index_assemble(gf_index* idx, uint32_t reserve);
gf_status gf_search_fullgraph(gf_index* idx, gf_plan* plan, const gf_search_params* params, uint32_t* ids_out,
                              float* dist_out, void* stream);

/*
 * Exact filtered k-NN: every point whose attributes lie inside the query's box competes;
 * squared L2 on the fp32 vectors; (distance, global id) order.  Replaces
 * naive_brute_force_with_filter (gpu_graph.cu:10782) and prefiltering_and_bruteforce
 * (brute_force.cuh:331).  Needs keep_fp32.  queries: device qnum x dim; lb/rb device.
 * Missing results are GF_NO_ID / +inf.
 */
gf_status gf_bruteforce(gf_index* idx, const float* queries, const float* lb, const float* rb, uint32_t qnum,
                        uint32_t k, uint32_t* ids_out, float* dist_out, void* stream);

/* Options of gf_bruteforce_ex (all zero = gf_bruteforce's behaviour). */
typedef struct {
    uint32_t path;       /* 0 = automatic: the tensor-core pass when the index has its fp16 tiles
                            (keep_fp32, dim <= 1024, finite rows) and k <= 128, else CUDA cores;
                            1 = CUDA cores only; 2 = tensor cores (GF_ERR_ARG when unavailable) */
    uint32_t test_fallback_every; /* 0 in normal use.  Test hook: queries whose index is a
                            multiple of this value skip the tensor-core proof and are answered
                            by the CUDA-core kernel, as unproven queries are */
    uint32_t test_wait;  /* 0 in normal use.  Test hook for the timeout path: every barrier wait
                            of the tensor-core pass gives up after test_wait polls and each query
                            tile's load expects 16 bytes more than it copies, so every CTA stops;
                            stats_out[1] counts them and all queries are answered by the CUDA-core
                            kernel (the results stay exact) */
    uint32_t* stats_out; /* optional device array of 3 words, written on the stream: queries
                            answered by the CUDA-core kernel after the tensor-core pass,
                            tensor-core waits that ran out (their queries are among the former),
                            and (128-query tile, 128-point tile) products multiplied */
} gf_bf_params;

/*
 * gf_bruteforce with options.  Same results on every path: on the tensor cores each query's
 * points are ranked by an fp16 product with a proven error bound, the 32 best are re-ranked
 * with the canonical fp32 distance, and a query whose result the bound cannot prove is
 * answered again by the CUDA-core kernel.  The dense query x point contraction replaces the
 * fp16 distance scan of prefiltering_and_bruteforce / dis_cal_reduce (brute_force.cuh:252-405).
 * Allocates its working memory on the stream (cudaMallocAsync).
 */
gf_status gf_bruteforce_ex(gf_index* idx, const float* queries, const float* lb, const float* rb, uint32_t qnum,
                           uint32_t k, uint32_t* ids_out, float* dist_out, const gf_bf_params* params, void* stream);

/*
 * Plan + search of one batch without allocating memory.  No counterpart in the
 * reference: it exists for callers that cannot allocate device memory at query time
 * (a latency-bound serving thread cannot absorb a cudaMalloc, which may synchronise the
 * device; a process whose device memory another allocator has already claimed has none
 * to give; an embedded caller may forbid allocation after start-up).  Same arguments and
 * results as gf_plan_queries followed by gf_search (queries, lb, rb, ids_out, dist_out
 * are device arrays the caller owns).  All working memory lives in one 4 MiB array of
 * device memory per GPU, reserved when the library is loaded and held until exit; a
 * batch that needs more (about 890 bytes per query at 128 dimensions and 16 cells)
 * returns GF_ERR_ARG.  The first call on a device looks up that array's device address
 * and should come before any stream capture.  Calls share the array: calls that overlap
 * on the GPU (different streams or threads) race and must be serialised by the caller.
 */
gf_status gf_search_noalloc(gf_index* idx, const float* queries, const float* lb, const float* rb, uint32_t qnum,
                            float prefilter, const gf_search_params* params, uint32_t* ids_out, float* dist_out,
                            void* stream);

/*
 * Spokesman assignment of the cross-edge compression (compress_global_graph_extreme,
 * tools.cuh:917-935): positions in cell order (cell c holds cell_sizes[c] points, rows of
 * `graphs` in that order, entries local ids); a point that is still its own spokesman
 * claims, in its graph row's order, every neighbour of higher position that is still its
 * own spokesman.  spokesman_out[pos] = the spokesman's position; rank_out[pos] (optional) =
 * the spokesman's rank among all spokesmen in position order (the reference's center_pos).
 */
gf_status gf_spokesman_host(uint32_t n, uint32_t n_cells, const uint32_t* cell_sizes, uint32_t degree,
                            const uint32_t* graphs, uint32_t* spokesman_out, uint32_t* rank_out,
                            uint32_t* n_spokesmen_out);

/* ------------------------------------------------------ file formats (host) */
/* Readers allocate with malloc; release with gf_free. */
void gf_free(void* p);

/* Compressed cross-cell graph (save_global_graph_extreme / load_global_graph_extreme,
 * tools.cuh:1012-1065): uint32 n, n_cells, E; n_cells spokesmen per cell; n_cells offsets
 * (prefix of the former); n ranks (center_pos, the spokesman rank of each position); then
 * n_cells x n_spokesmen x E local ids: block c holds the spokesmen's E edges into cell c. */
gf_status gf_write_spokesman_graph(const char* path, uint32_t n, uint32_t n_cells, uint32_t e,
                                   const uint32_t* center_num, const uint32_t* col_offset, const uint32_t* center_pos,
                                   const uint32_t* edges);
gf_status gf_read_spokesman_graph(const char* path, uint32_t* n, uint32_t* n_cells, uint32_t* e, uint32_t** center_num,
                                  uint32_t** col_offset, uint32_t** center_pos, uint32_t** edges);

/* .fvecs: per row int32 d then d float32 (tools.cuh:85-106). */
gf_status gf_read_fvecs(const char* path, float** data, uint32_t* n, uint32_t* dim);
gf_status gf_write_fvecs(const char* path, const float* data, uint32_t n, uint32_t dim);
/* u8bin: uint32 n, uint32 d, n*d uint8 (tools.cuh:108-150). */
gf_status gf_read_u8bin(const char* path, uint8_t** data, uint32_t* n, uint32_t* dim);
/* .q file: uint32 n, uint32 d, d float32 scales, d int32 zero points, n*d int8 codes
 * (save_dataset_quantified / load_dataset_quantified, production_adapter.cuh:240-285).
 * The reader allocates three arrays (gf_free each). */
gf_status gf_read_q(const char* path, int8_t** codes, float** scales, int32_t** zero_points, uint32_t* n,
                    uint32_t* dim);
gf_status gf_write_q(const char* path, const int8_t* codes, const float* scales, const int32_t* zero_points,
                     uint32_t n, uint32_t dim);
/*
 * Per-dimension affine int8 quantisation of data * alpha (the reference's host quantiser,
 * production_adapter.cuh:316-337; its device kernel integer_production_kernal, :8-47,
 * computes the same with round-half-even).  scale = (max - min) / 255, zero_point =
 * round(-128 - min / scale), q = round(x / scale) + zero_point, both clamped to
 * [-128, 127], round half away from zero, min / max starting from 100000 / -100000; a
 * constant dimension gets scale 1.  gf_quantize_i8: device arrays (data n x dim, q_out
 * n x dim, scales_out and zero_points_out dim), synchronises `stream`; _host: host arrays
 * (q_out may be NULL to compute only the parameters).
 */
gf_status gf_quantize_i8(const float* data, uint32_t n, uint32_t dim, float alpha, int8_t* q_out, float* scales_out,
                         int32_t* zero_points_out, void* stream);
gf_status gf_quantize_i8_host(const float* data, uint32_t n, uint32_t dim, float alpha, int8_t* q_out,
                              float* scales_out, int32_t* zero_points_out);
/* attrs.bin: uint32 n, uint32 a, n*a int32 (tools.cuh:747-765). */
gf_status gf_read_attrs(const char* path, int32_t** attrs, uint32_t* n, uint32_t* a);
gf_status gf_write_attrs(const char* path, const int32_t* attrs, uint32_t n, uint32_t a);
/* graph / global graph / result blob: uint32 n, uint32 k, n*k uint32 (tools.cuh:205-223;
 * the per-cell .cagraN files use the same header with int32 fields). */
gf_status gf_read_u32mat(const char* path, uint32_t** data, uint32_t* n, uint32_t* k);
gf_status gf_write_u32mat(const char* path, const uint32_t* data, uint32_t n, uint32_t k);
/* range file: per query per attribute int32 l, int32 r, no header (tools.cuh:275-291). */
gf_status gf_read_ranges(const char* path, uint32_t qnum, uint32_t a, int32_t* l_out, int32_t* r_out);
gf_status gf_write_ranges(const char* path, const int32_t* l, const int32_t* r, uint32_t qnum, uint32_t a);
/* cluster.bin: int32 n, n int32 labels (tools.cuh:547-567). */
gf_status gf_read_labels(const char* path, int32_t** labels, uint32_t* n);
/*
 * grid_info: int32 N, int32 a, int32 grid[a]; per dim int32 l_quant[g], r_quant[g],
 * pid_list[N]; then int32 global_pid[N] (real_dataset_adapter.cuh:563-586).
 * quant arrays: sum(grid) entries; cell_of: N.  Outputs are malloc'd.
 */
gf_status gf_read_grid(const char* path, uint32_t* n, uint32_t* a, uint32_t** grid, int32_t** l_quant,
                       int32_t** r_quant, uint32_t** cell_of);

#ifdef __cplusplus
}
#endif
#endif
