// Internal declarations shared by the garfield_b200 translation units.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/garfield.h"

namespace gf {

constexpr uint32_t kEmpty = 0xFFFFFFFFu;
constexpr uint32_t kExplored = 0x80000000u;  // list entry already expanded
constexpr uint32_t kInRange = 0x40000000u;   // point satisfies the query box
constexpr uint32_t kPosMask = 0x3FFFFFFFu;   // cell-major position (< 2^30 points)
constexpr uint32_t kMaxAttr = 8;
constexpr uint32_t kHopSlots = 64;  // list entries that seed a cross-cell hop (gpu_graph.cu:3569)

void set_error(const std::string& msg);
gf_status fail(gf_status s, const std::string& msg);
gf_status cuda_fail(cudaError_t e, const char* what);

#define GF_CUDA(call)                                    \
    do {                                                 \
        cudaError_t e_ = (call);                         \
        if (e_ != cudaSuccess) return gf::cuda_fail(e_, #call); \
    } while (0)

// Device-resident index in cell-major order: point positions seg[c] .. seg[c+1]-1
// belong to cell c, in increasing global id (the reference's "logical position",
// offset[pid] + local_idx, tools.cuh:862-889).
// Geometry of the attribute tiles (gf_bf_tc.cu attr_tiles_prepare): rows of the index in
// the Morton order of their attributes, kTileRows per tile, kSuperTiles tiles per
// super-tile.  The box counts and the search's exact route walk them one warp per query,
// one lane per tile of a super-tile and 32 rows of a tile per step.
constexpr uint32_t kTileRows = 128;
constexpr uint32_t kSuperTiles = 32;
static_assert(kSuperTiles == 32, "one lane per tile of a super-tile");
static_assert(kTileRows % 32 == 0, "tiles are walked 32 rows at a time");

struct DeviceIndex {
    int device = 0;
    uint32_t n = 0, dim = 0, d8 = 0, d4 = 0, a = 0, ncells = 0, degree = 0, E = 0, C = 0;
    float alpha = 1.0f;
    uint32_t min_cell = 0;
    std::vector<uint32_t> grid;       // a
    std::vector<float> lq, rq;        // sum(grid)
    std::vector<uint32_t> seg_h;      // ncells + 1
    std::vector<uint32_t> entry_h;    // deterministic entry local ids
    uint64_t bytes = 0;
    // device arrays
    uint4* vec16 = nullptr;      // n x d8 halves (alpha-scaled), as 16-byte chunks (codec 0)
    // byte codecs (codec 1 = int8, 2 = uint8): rows of d16 bytes, decoded scale * (q - zp)
    uint32_t codec = 0, d16 = 0;
    uint4* vec8 = nullptr;       // rows x d16 bytes
    float* csc = nullptr;        // d16 per-element -scale (0 past dim)
    float* cbi = nullptr;        // d16 per-element 2^23 + bias (bias = zp + 128 for int8, zp for uint8)
    std::vector<float> scales_h; // dim
    std::vector<int32_t> zps_h;  // dim
    float4* vec32 = nullptr;     // n x d4 fp32 (optional)
    float* attrs = nullptr;      // n x a
    uint32_t* graph = nullptr;   // n x degree positions (NULL when host_graph)
    uint32_t* cross = nullptr;   // cross_rows x (ncells*E) positions (NULL when host_graph)
    uint32_t cross_rows = 0;     // n, or the number of spokesmen (cross_spokesman)
    std::vector<uint32_t> spk_start_h;  // cross_spokesman: first spokesman rank of each cell (ncells + 1)
    uint32_t* spk_rank = nullptr; // n: row of each position's cross edges (spokesman rank), or NULL
    // full-graph ablation (gf_index_assemble): n x fdeg positions, entry positions
    uint32_t* fgraph = nullptr;
    uint32_t fdeg = 0, fentry_n = 0;
    uint32_t* fentry = nullptr;
    std::vector<uint32_t> fentry_h;
    // host_graph: graphs and cross edges stay in pinned host memory and are copied to the
    // device per batch of cells (gf_search_batched)
    bool host_graph = false;
    uint32_t* graph_h = nullptr; // pinned, n x degree positions (position order)
    uint32_t* cross_h = nullptr; // pinned, ncells x cross_rows x E: [target cell][source row][edge] (rows:
                                 // positions, or spokesman ranks with cross_spokesman)
    // shard: the device holds the vectors, graph rows and cross blocks of shard_cells only
    // (compact, in shard order); positions, attributes and ids stay global
    bool sharded = false;
    std::vector<uint32_t> shard_cells;
    uint32_t n_stored = 0;         // vector / graph rows held
    int32_t* sh_slot = nullptr;    // ncells: shard slot of each cell, -1 = not held
    long long* sh_gofs = nullptr;  // per slot: graph element offset of the cell's first row
    long long* sh_xofs = nullptr;  // slot x slot: cross block offset [target][source]
    long long* sh_vsh = nullptr;   // per slot: vector row - position
    uint32_t* i2g = nullptr;     // position -> global id
    uint32_t* seg = nullptr;     // ncells + 1
    uint32_t* grid_d = nullptr;  // a
    float* lq_d = nullptr;
    float* rq_d = nullptr;
    float* centroids = nullptr;  // C x dim fp32
    float* cnorm = nullptr;      // C x (|c - m|^2, |c - m|) of the centroids (tensor-core planner)
    float* cmean = nullptr;      // dim: the centroids' mean m (tensor-core planner)
    uint32_t* hist = nullptr;    // ncells x C
    uint32_t* entry = nullptr;   // entry_h on device
    // tensor-core brute force (gf_bf_tc.cu): centred, scaled fp16 copy of the fp32 rows in
    // 128-point tcgen05 tiles, per point (1 - kappa)|x~|^2, per tile attribute bounds
    bool bf_ok = false;
    bool at_ok = false;          // attribute tiles (bf_tbox, bf_attrs, bf_rowpos, bf_tcnt) built
    bool cells_hold_rows = false; // every row's attributes lie in its cell's slice ranges
    uint32_t* bf_tcnt = nullptr; // bf_tiles: points of each tile whose attributes are all numbers
    uint32_t bf_stiles = 0;      // super-tiles: 32 consecutive tiles (box counts)
    float* bf_sbox = nullptr;    // bf_stiles x 2 x a8: attribute bounds per super-tile
    uint32_t* bf_scnt = nullptr; // bf_stiles: sum of the super-tile's bf_tcnt
    uint32_t bf_dp = 0, bf_tiles = 0;   // padded row length (multiple of 16), point tiles
    float bf_scale = 1.0f, bf_dmax = 0.0f;  // power-of-two scale s, largest residual |x - x^|
    void* bf_x = nullptr;        // bf_tiles x 128 x bf_dp halves
    float* bf_px = nullptr;      // bf_tiles x 128 (+inf past n)
    float* bf_mean = nullptr;    // dim
    float* bf_tbox = nullptr;    // bf_tiles x 2 x a8: attribute bounds per tile (a8 = a rounded up to 4)
    float* bf_attrs = nullptr;   // bf_tiles x 128 x a (NaN past n)
    uint32_t* bf_rowpos = nullptr; // bf_tiles x 128: position of each row (rows in attribute Morton order)
    float* bf_arange = nullptr;  // 2 x a: attribute origin and inverse extent (Morton codes)
    // working memory of gf_bruteforce, kept between calls and grown on demand; the event
    // orders calls on different streams, the mutex guards the buffer's replacement
    void* bf_ws = nullptr;
    size_t bf_ws_bytes = 0;
    cudaEvent_t bf_ws_ev = nullptr;
    std::shared_ptr<std::mutex> bf_mu = std::make_shared<std::mutex>();
};

struct BatchState;  // gf_batch.cu: buffers, streams and events of gf_search_batched
void free_batch_state(BatchState* b);

struct Plan {
    gf_index* idx = nullptr;
    int device = 0;  // the index's device, kept so that destroying the plan never reads the index
    uint32_t max_q = 0, qnum = 0;
    bool planned = false;
    float prefilter = 0.0f;
    cudaStream_t stream = nullptr;
    // device buffers
    uint4* q16 = nullptr;        // max_q x d8 halves
    float* q32 = nullptr;        // max_q x dim (copy of the fp32 queries)
    float* lb = nullptr;         // max_q x a
    float* rb = nullptr;
    uint32_t* counts = nullptr;  // max_q
    uint32_t* offsets = nullptr; // max_q
    uint32_t* cells = nullptr;   // max_q x ncells
    uint32_t* top4 = nullptr;    // max_q x 4
    float* S = nullptr;          // max_q x centroid_tc_stride query-centroid products (tensor-core planner), or NULL
    float* part_d = nullptr;     // max_q x splits x 4 per-range centroid candidates
    uint32_t* part_i = nullptr;
    uint32_t* box = nullptr;     // max_q (box counts)
    uint32_t* task = nullptr;    // max_q processing order
    uint32_t* scratch = nullptr; // small counters: [0] queue head, [1..] histogram
    unsigned long long* stats = nullptr;  // 8 counters
    void* scan_tmp = nullptr;
    size_t scan_tmp_bytes = 0;
    // device copies of gf_search_host's inputs and outputs; grown on demand, kept
    // between calls so that steady-state calls allocate nothing
    void* io = nullptr;
    size_t io_bytes = 0;
    BatchState* batch = nullptr;  // created by the first gf_search_batched
    unsigned long long* run = nullptr;  // running keys of searches on a shard index
    uint32_t* xmark = nullptr;          // max_q: queries answered by the tensor-core exact scan (exact_tc)
    // shard indexes: live[0] = queries with two or more of the shard's cells, live[1..] their
    // ids; lq32 their fp32 rows, gathered for the centroid planner
    uint32_t* live = nullptr;
    float* lq32 = nullptr;
    // side stream of the centroid stage (whole indexes; null: everything on the caller's stream)
    cudaStream_t side = nullptr;
    cudaEvent_t ev_fork = nullptr, ev_join = nullptr;
    // pinned: the timeout counters of the last gf_search_host, read back with its results
    unsigned long long* flags_h = nullptr;
    size_t run_cap = 0;
};

}  // namespace gf

struct gf_index {
    gf::DeviceIndex d;
};

struct gf_plan {
    gf::Plan p;
};

namespace gf {
// gf_plan.cu
uint32_t centroid_splits(uint32_t C);  // centroid ranges of the top-4 kernel
uint32_t centroid_chunk(uint32_t C);   // centroids per range (multiple of 128)
gf_status plan_queries(gf_index* idx, gf_plan* plan, const float* queries, const float* lb, const float* rb,
                       uint32_t qnum, float prefilter, cudaStream_t s);
// Significant bits of a query's cell count (0..ncells): the task-order radix sort reads only
// these, one pass per 8 bits instead of four for the whole word; the order is the same.
inline int count_sort_bits(uint32_t ncells) {
    int b = 1;
    while (b < 32 && (ncells >> b)) ++b;
    return b;
}
// gf_centroid_tc.cu
bool centroid_tc_usable(const DeviceIndex& d);
size_t centroid_tc_stride(const DeviceIndex& d);  // floats per row of the plan's S
// live (nullable, device): live[0] rows of q32 in use, row j being query live[1 + j]
gf_status centroid_top4_tc(const DeviceIndex& d, const float* q32, uint32_t qnum, float* S, uint32_t* top4,
                           uint32_t* counters, cudaStream_t s, const uint32_t* live = nullptr);
// gf_search.cu
// Restriction of one search launch to a set of cells ("slots"), whose graph rows and
// cross-edge rows may lie anywhere in device memory (batched and out-of-core search).
// Row of position pos (cell c, slot b = slot[c]): graph + gofs[b] + (pos - seg[c]) * R.
// Cross edges of source pos (cell s) toward cell t: cross + xofs[slot[t] * nslots +
// slot[s]] + (pos - seg[s]) * xstride.  Vector rows: pos + vsh[slot[c]].
// Each query's results are merged into run[q]
// (k keys, sorted) instead of being written as ids.
struct CellView {
    const int32_t* slot = nullptr;    // device, ncells; -1 = cell not searched
    const long long* gofs = nullptr;  // device, nslots
    const long long* xofs = nullptr;  // device, nslots x nslots
    const long long* vsh = nullptr;   // device, nslots: vector row = pos + vsh[slot] (NULL: pos)
    const uint32_t* graph = nullptr;
    const uint32_t* cross = nullptr;
    uint32_t nslots = 0, xstride = 0;
    unsigned long long* run = nullptr;  // device, qnum x k
    bool accumulate_stats = false;      // add to the plan's counters instead of resetting them
};
gf_status search(gf_index* idx, gf_plan* plan, const gf_search_params* prm, uint32_t* ids, float* dist,
                 cudaStream_t s, const CellView* view = nullptr, bool fullgraph = false);
CellView shard_view(const DeviceIndex& d);
// run keys -> ids (via position -> global id) and distances
gf_status finish_run(gf_index* idx, const unsigned long long* run, uint32_t total, uint32_t* ids, float* dist,
                     cudaStream_t s);
// gf_bruteforce.cu
// qmask (device, qnum words, or NULL): only queries q with qmask[q] != 0 are answered (tensor-core
// path only); the others' rows of ids / dist are left untouched
gf_status bruteforce(gf_index* idx, const float* queries, const float* lb, const float* rb, uint32_t qnum,
                     uint32_t k, uint32_t* ids, float* dist, cudaStream_t s, const gf_bf_params* prm = nullptr,
                     const uint32_t* qmask = nullptr);
// gf_bf_tc.cu
gf_status attr_tiles_prepare(DeviceIndex& d);  // at index creation, after attrs
gf_status bf_tc_prepare(DeviceIndex& d);  // at index creation, after vec32 and attr_tiles_prepare
// plan box counts from the attribute tiles (d.at_ok); same counts as testing every point.
// coarse: an estimate without the row scan (points of tiles inside the box, plus half of the
// points of each tile that meets it only in part), for the search's cost rule
void box_count_tiles(const DeviceIndex& d, const float* lb, const float* rb, uint32_t qnum, uint32_t* box,
                     cudaStream_t s, bool coarse = false);
void free_bf_tc(DeviceIndex& d);
bool bf_tc_usable(const DeviceIndex& d, uint32_t k);
// Tensor-core pass: writes the proven queries' results and appends the others to
// fb_list / fb_cnt (answered afterwards by the CUDA-core kernel).
size_t bf_tc_ws_bytes(const DeviceIndex& d, uint32_t qnum, uint32_t k);  // working memory of bf_tc_run
gf_status bf_tc_run(gf_index* idx, const float* queries, const float* lb, const float* rb, uint32_t qnum, uint32_t k,
                    uint32_t* ids, float* dist, void* ws, uint32_t* fb_list, uint32_t* fb_cnt, uint32_t test_every,
                    uint32_t test_wait, uint32_t* timeouts, uint32_t* products, cudaStream_t s,
                    const uint32_t* qmask = nullptr);
// gf_index.cu: greedy spokesman assignment (compress_global_graph_extreme, tools.cuh:917-935);
// graphs: n x degree local ids, rows in position (cell) order
void spokesman_assign(uint32_t n, uint32_t n_cells, const uint32_t* cell_sizes, uint32_t degree,
                      const uint32_t* graphs, uint32_t* spk, uint32_t* rank, uint32_t* n_spk);
// gf_codec.cu
void quantize_i8_host(const float* data, uint32_t n, uint32_t dim, float alpha, int8_t* q, float* scales,
                      int32_t* zps);
// gf_index.cu
void launch_f2h(const float* in, uint32_t n, uint32_t dim, uint32_t d8, float alpha, uint4* out, cudaStream_t s);
}  // namespace gf
