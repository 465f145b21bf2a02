// Readers and writers for the reference's on-disk formats, and gf_index_open.
// Every reader checks the file size against its header and returns GF_ERR_IO /
// GF_ERR_FORMAT instead of exiting (the reference prints and calls exit(-1),
// tools.cuh:66,207).
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "gf_internal.h"

using gf::fail;

namespace {

struct File {
    FILE* f = nullptr;
    ~File() {
        if (f) fclose(f);
    }
};

gf_status open_read(File& fl, const char* path, long long* size) {
    if (!path) return fail(GF_ERR_ARG, "null path");
    fl.f = fopen(path, "rb");
    if (!fl.f) return fail(GF_ERR_IO, std::string("cannot open ") + path);
    if (fseeko(fl.f, 0, SEEK_END) != 0) return fail(GF_ERR_IO, std::string("cannot seek ") + path);
    *size = (long long)ftello(fl.f);
    fseeko(fl.f, 0, SEEK_SET);
    return GF_OK;
}

gf_status rd(File& fl, void* dst, size_t bytes, const char* path) {
    if (bytes && fread(dst, 1, bytes, fl.f) != bytes) return fail(GF_ERR_FORMAT, std::string("short read ") + path);
    return GF_OK;
}

gf_status open_write(File& fl, const char* path) {
    if (!path) return fail(GF_ERR_ARG, "null path");
    fl.f = fopen(path, "wb");
    if (!fl.f) return fail(GF_ERR_IO, std::string("cannot create ") + path);
    return GF_OK;
}

gf_status wr(File& fl, const void* src, size_t bytes, const char* path) {
    if (bytes && fwrite(src, 1, bytes, fl.f) != bytes) return fail(GF_ERR_IO, std::string("short write ") + path);
    return GF_OK;
}

template <typename T>
T* xmalloc(size_t count) {
    return static_cast<T*>(malloc(std::max<size_t>(count, 1) * sizeof(T)));
}

#define TRY(x)                       \
    do {                             \
        gf_status s_ = (x);          \
        if (s_ != GF_OK) return s_;  \
    } while (0)

// Frees every malloc'd reader output at scope exit.
struct Holder {
    std::vector<void*> v;
    ~Holder() {
        for (void* p : v) free(p);
    }
    template <typename T>
    T* keep(T* p) {
        v.push_back((void*)p);
        return p;
    }
};

}  // namespace

extern "C" {

void gf_free(void* p) { free(p); }

gf_status gf_read_fvecs(const char* path, float** data, uint32_t* n, uint32_t* dim) {
    File fl;
    long long size;
    TRY(open_read(fl, path, &size));
    int32_t d;
    if (size < 4) return fail(GF_ERR_FORMAT, "empty fvecs");
    TRY(rd(fl, &d, 4, path));
    if (d <= 0) return fail(GF_ERR_FORMAT, "bad fvecs dimension");
    long long row = 4LL * (d + 1);
    if (size % row != 0) return fail(GF_ERR_FORMAT, "fvecs size not a multiple of the row size");
    uint32_t num = (uint32_t)(size / row);
    float* out = xmalloc<float>((size_t)num * d);
    if (!out) return fail(GF_ERR_OOM, "host allocation");
    fseeko(fl.f, 0, SEEK_SET);
    for (uint32_t i = 0; i < num; ++i) {
        int32_t di;
        if (rd(fl, &di, 4, path) != GF_OK || di != d || rd(fl, out + (size_t)i * d, 4ull * d, path) != GF_OK) {
            free(out);
            return fail(GF_ERR_FORMAT, "fvecs row dimension mismatch");
        }
    }
    *data = out;
    *n = num;
    *dim = (uint32_t)d;
    return GF_OK;
}

gf_status gf_write_fvecs(const char* path, const float* data, uint32_t n, uint32_t dim) {
    File fl;
    TRY(open_write(fl, path));
    int32_t d = (int32_t)dim;
    for (uint32_t i = 0; i < n; ++i) {
        TRY(wr(fl, &d, 4, path));
        TRY(wr(fl, data + (size_t)i * dim, 4ull * dim, path));
    }
    return GF_OK;
}

gf_status gf_read_u8bin(const char* path, uint8_t** data, uint32_t* n, uint32_t* dim) {
    File fl;
    long long size;
    TRY(open_read(fl, path, &size));
    uint32_t h[2];
    TRY(rd(fl, h, 8, path));
    if ((long long)h[0] * h[1] + 8 != size) return fail(GF_ERR_FORMAT, "u8bin size mismatch");
    uint8_t* out = xmalloc<uint8_t>((size_t)h[0] * h[1]);
    if (!out) return fail(GF_ERR_OOM, "host allocation");
    if (rd(fl, out, (size_t)h[0] * h[1], path) != GF_OK) {
        free(out);
        return GF_ERR_FORMAT;
    }
    *data = out;
    *n = h[0];
    *dim = h[1];
    return GF_OK;
}

// .q file (save_dataset_quantified / load_dataset_quantified, production_adapter.cuh:240-285):
// uint32 n, uint32 d, d x float32 scales, d x int32 zero points, n*d int8 codes.
gf_status gf_read_q(const char* path, int8_t** codes, float** scales, int32_t** zero_points, uint32_t* n,
                    uint32_t* dim) {
    File fl;
    long long size;
    TRY(open_read(fl, path, &size));
    uint32_t h[2];
    TRY(rd(fl, h, 8, path));
    if (h[1] == 0 || 8 + 8ll * h[1] + (long long)h[0] * h[1] != size) return fail(GF_ERR_FORMAT, ".q size mismatch");
    float* sc = xmalloc<float>(h[1]);
    int32_t* zp = xmalloc<int32_t>(h[1]);
    int8_t* q = xmalloc<int8_t>(std::max<size_t>((size_t)h[0] * h[1], 1));
    if (!sc || !zp || !q) {
        free(sc);
        free(zp);
        free(q);
        return fail(GF_ERR_OOM, "host allocation");
    }
    if (rd(fl, sc, 4ull * h[1], path) != GF_OK || rd(fl, zp, 4ull * h[1], path) != GF_OK ||
        rd(fl, q, (size_t)h[0] * h[1], path) != GF_OK) {
        free(sc);
        free(zp);
        free(q);
        return GF_ERR_FORMAT;
    }
    *codes = q;
    *scales = sc;
    *zero_points = zp;
    *n = h[0];
    *dim = h[1];
    return GF_OK;
}

gf_status gf_write_q(const char* path, const int8_t* codes, const float* scales, const int32_t* zero_points,
                     uint32_t n, uint32_t dim) {
    File fl;
    TRY(open_write(fl, path));
    uint32_t h[2] = {n, dim};
    TRY(wr(fl, h, 8, path));
    TRY(wr(fl, scales, 4ull * dim, path));
    TRY(wr(fl, zero_points, 4ull * dim, path));
    TRY(wr(fl, codes, (size_t)n * dim, path));
    return GF_OK;
}

gf_status gf_read_attrs(const char* path, int32_t** attrs, uint32_t* n, uint32_t* a) {
    File fl;
    long long size;
    TRY(open_read(fl, path, &size));
    uint32_t h[2];
    TRY(rd(fl, h, 8, path));
    if (8 + 4LL * h[0] * h[1] != size) return fail(GF_ERR_FORMAT, "attrs size mismatch");
    int32_t* out = xmalloc<int32_t>((size_t)h[0] * h[1]);
    if (!out) return fail(GF_ERR_OOM, "host allocation");
    if (rd(fl, out, 4ull * h[0] * h[1], path) != GF_OK) {
        free(out);
        return GF_ERR_FORMAT;
    }
    *attrs = out;
    *n = h[0];
    *a = h[1];
    return GF_OK;
}

gf_status gf_write_attrs(const char* path, const int32_t* attrs, uint32_t n, uint32_t a) {
    File fl;
    TRY(open_write(fl, path));
    uint32_t h[2] = {n, a};
    TRY(wr(fl, h, 8, path));
    return wr(fl, attrs, 4ull * n * a, path);
}

gf_status gf_read_u32mat(const char* path, uint32_t** data, uint32_t* n, uint32_t* k) {
    File fl;
    long long size;
    TRY(open_read(fl, path, &size));
    uint32_t h[2];
    TRY(rd(fl, h, 8, path));
    if (8 + 4LL * h[0] * h[1] != size) return fail(GF_ERR_FORMAT, std::string("matrix size mismatch ") + path);
    uint32_t* out = xmalloc<uint32_t>((size_t)h[0] * h[1]);
    if (!out) return fail(GF_ERR_OOM, "host allocation");
    if (rd(fl, out, 4ull * h[0] * h[1], path) != GF_OK) {
        free(out);
        return GF_ERR_FORMAT;
    }
    *data = out;
    *n = h[0];
    *k = h[1];
    return GF_OK;
}

gf_status gf_write_u32mat(const char* path, const uint32_t* data, uint32_t n, uint32_t k) {
    File fl;
    TRY(open_write(fl, path));
    uint32_t h[2] = {n, k};
    TRY(wr(fl, h, 8, path));
    return wr(fl, data, 4ull * n * k, path);
}

gf_status gf_write_spokesman_graph(const char* path, uint32_t n, uint32_t n_cells, uint32_t e,
                                   const uint32_t* center_num, const uint32_t* col_offset, const uint32_t* center_pos,
                                   const uint32_t* edges) {
    if (!center_num || !col_offset || !center_pos || !edges) return fail(GF_ERR_ARG, "null array");
    uint64_t total = 0;
    for (uint32_t c = 0; c < n_cells; ++c) total += center_num[c];
    File fl;
    TRY(open_write(fl, path));
    uint32_t h[3] = {n, n_cells, e};
    TRY(wr(fl, h, 12, path));
    TRY(wr(fl, center_num, 4ull * n_cells, path));
    TRY(wr(fl, col_offset, 4ull * n_cells, path));
    TRY(wr(fl, center_pos, 4ull * n, path));
    return wr(fl, edges, 4ull * total * e * n_cells, path);
}

gf_status gf_read_spokesman_graph(const char* path, uint32_t* n, uint32_t* n_cells, uint32_t* e, uint32_t** center_num,
                                  uint32_t** col_offset, uint32_t** center_pos, uint32_t** edges) {
    File fl;
    long long size;
    TRY(open_read(fl, path, &size));
    uint32_t h[3];
    if (size < 12) return fail(GF_ERR_FORMAT, std::string("compressed graph too short ") + path);
    TRY(rd(fl, h, 12, path));
    const uint64_t head = 12 + 8ull * h[1] + 4ull * h[0];
    if ((uint64_t)size < head) return fail(GF_ERR_FORMAT, std::string("compressed graph too short ") + path);
    std::vector<uint32_t> cn(h[1]), co(h[1]);
    TRY(rd(fl, cn.data(), 4ull * h[1], path));
    TRY(rd(fl, co.data(), 4ull * h[1], path));
    uint64_t total = 0;
    for (uint32_t c = 0; c < h[1]; ++c) {
        if (co[c] != total) return fail(GF_ERR_FORMAT, std::string("compressed graph offsets ") + path);
        total += cn[c];
    }
    if ((uint64_t)size != head + 4ull * total * h[2] * h[1])
        return fail(GF_ERR_FORMAT, std::string("compressed graph size mismatch ") + path);
    uint32_t* a = xmalloc<uint32_t>(h[1]);
    uint32_t* b = xmalloc<uint32_t>(h[1]);
    uint32_t* c = xmalloc<uint32_t>(h[0]);
    uint32_t* d = xmalloc<uint32_t>((size_t)total * h[2] * h[1]);
    if (!a || !b || !c || !d) {
        free(a), free(b), free(c), free(d);
        return fail(GF_ERR_OOM, "host allocation");
    }
    std::memcpy(a, cn.data(), 4ull * h[1]);
    std::memcpy(b, co.data(), 4ull * h[1]);
    if (rd(fl, c, 4ull * h[0], path) != GF_OK || rd(fl, d, 4ull * total * h[2] * h[1], path) != GF_OK) {
        free(a), free(b), free(c), free(d);
        return GF_ERR_FORMAT;
    }
    for (uint32_t i = 0; i < h[0]; ++i)
        if (c[i] >= total) {
            free(a), free(b), free(c), free(d);
            return fail(GF_ERR_FORMAT, std::string("spokesman rank out of range ") + path);
        }
    *n = h[0];
    *n_cells = h[1];
    *e = h[2];
    *center_num = a;
    *col_offset = b;
    *center_pos = c;
    *edges = d;
    return GF_OK;
}

gf_status gf_spokesman_host(uint32_t n, uint32_t n_cells, const uint32_t* cell_sizes, uint32_t degree,
                            const uint32_t* graphs, uint32_t* spokesman_out, uint32_t* rank_out,
                            uint32_t* n_spokesmen_out) {
    if (!cell_sizes || !graphs || !spokesman_out) return fail(GF_ERR_ARG, "null array");
    uint64_t sum = 0;
    for (uint32_t c = 0; c < n_cells; ++c) sum += cell_sizes[c];
    if (sum != n) return fail(GF_ERR_ARG, "cell sizes do not add up to n");
    gf::spokesman_assign(n, n_cells, cell_sizes, degree, graphs, spokesman_out, rank_out, n_spokesmen_out);
    return GF_OK;
}

gf_status gf_read_ranges(const char* path, uint32_t qnum, uint32_t a, int32_t* l_out, int32_t* r_out) {
    File fl;
    long long size;
    TRY(open_read(fl, path, &size));
    if (size < 8LL * qnum * a) return fail(GF_ERR_FORMAT, "range file shorter than qnum x attrs");
    std::vector<int32_t> buf((size_t)qnum * a * 2);
    TRY(rd(fl, buf.data(), buf.size() * 4, path));
    for (uint32_t q = 0; q < qnum; ++q)
        for (uint32_t j = 0; j < a; ++j) {
            l_out[q * a + j] = buf[(size_t)q * a * 2 + j * 2];
            r_out[q * a + j] = buf[(size_t)q * a * 2 + j * 2 + 1];
        }
    return GF_OK;
}

gf_status gf_write_ranges(const char* path, const int32_t* l, const int32_t* r, uint32_t qnum, uint32_t a) {
    File fl;
    TRY(open_write(fl, path));
    std::vector<int32_t> buf((size_t)qnum * a * 2);
    for (uint32_t q = 0; q < qnum; ++q)
        for (uint32_t j = 0; j < a; ++j) {
            buf[(size_t)q * a * 2 + j * 2] = l[q * a + j];
            buf[(size_t)q * a * 2 + j * 2 + 1] = r[q * a + j];
        }
    return wr(fl, buf.data(), buf.size() * 4, path);
}

gf_status gf_read_labels(const char* path, int32_t** labels, uint32_t* n) {
    File fl;
    long long size;
    TRY(open_read(fl, path, &size));
    int32_t num;
    TRY(rd(fl, &num, 4, path));
    if (num < 0 || 4 + 4LL * num != size) return fail(GF_ERR_FORMAT, "cluster file size mismatch");
    int32_t* out = xmalloc<int32_t>((size_t)num);
    if (!out) return fail(GF_ERR_OOM, "host allocation");
    if (rd(fl, out, 4ull * num, path) != GF_OK) {
        free(out);
        return GF_ERR_FORMAT;
    }
    *labels = out;
    *n = (uint32_t)num;
    return GF_OK;
}

gf_status gf_read_grid(const char* path, uint32_t* n, uint32_t* a, uint32_t** grid, int32_t** l_quant,
                       int32_t** r_quant, uint32_t** cell_of) {
    File fl;
    long long size;
    TRY(open_read(fl, path, &size));
    int32_t h[2];
    TRY(rd(fl, h, 8, path));
    if (h[0] <= 0 || h[1] <= 0 || h[1] > (int32_t)gf::kMaxAttr) return fail(GF_ERR_FORMAT, "bad grid header");
    uint32_t num = (uint32_t)h[0], dims = (uint32_t)h[1];
    std::vector<int32_t> g(dims);
    TRY(rd(fl, g.data(), 4ull * dims, path));
    long long total = 0, expect = 8 + 4LL * dims;
    for (uint32_t j = 0; j < dims; ++j) {
        if (g[j] <= 0) return fail(GF_ERR_FORMAT, "bad grid size");
        total += g[j];
        expect += 4LL * (2LL * g[j] + num);
    }
    expect += 4LL * num;
    if (expect != size) return fail(GF_ERR_FORMAT, "grid file size mismatch");
    uint32_t* go = xmalloc<uint32_t>(dims);
    int32_t* lo = xmalloc<int32_t>((size_t)total);
    int32_t* ro = xmalloc<int32_t>((size_t)total);
    uint32_t* co = xmalloc<uint32_t>(num);
    std::vector<int32_t> pid(num);
    gf_status st = GF_OK;
    size_t off = 0;
    for (uint32_t j = 0; j < dims && st == GF_OK; ++j) {
        go[j] = (uint32_t)g[j];
        st = rd(fl, lo + off, 4ull * g[j], path);
        if (st == GF_OK) st = rd(fl, ro + off, 4ull * g[j], path);
        if (st == GF_OK) st = rd(fl, pid.data(), 4ull * num, path);  // per-dim slice ids (unused)
        off += g[j];
    }
    if (st == GF_OK) st = rd(fl, co, 4ull * num, path);
    if (st != GF_OK) {
        free(go);
        free(lo);
        free(ro);
        free(co);
        return st;
    }
    *n = num;
    *a = dims;
    *grid = go;
    *l_quant = lo;
    *r_quant = ro;
    *cell_of = co;
    return GF_OK;
}

// Load the reference's index files (realdataset_search.cu:2118-2393) and build the index.
gf_status gf_index_open(const gf_index_files* fs, int device, gf_index** out) {
    if (!fs || !out) return fail(GF_ERR_ARG, "null argument");
    Holder hold;
    float* vec = nullptr;
    uint32_t n = 0, dim = 0;
    uint8_t* u8 = nullptr;
    if (fs->codec == 2) {  // u8bin data (load_data_u8, tools.cuh:108-150); fp32 copy for the planner
        TRY(gf_read_u8bin(fs->data_path, &u8, &n, &dim));
        hold.keep(u8);
        vec = xmalloc<float>(std::max<size_t>((size_t)n * dim, 1));
        if (!vec) return fail(GF_ERR_OOM, "host allocation");
        for (size_t i = 0; i < (size_t)n * dim; ++i) vec[i] = (float)u8[i];
    } else {
        TRY(gf_read_fvecs(fs->data_path, &vec, &n, &dim));
    }
    hold.keep(vec);
    int8_t* qcodes = nullptr;
    float* qscales = nullptr;
    int32_t* qzps = nullptr;
    if (fs->codec == 1 && fs->quantized) {
        uint32_t qn = 0, qd = 0;
        TRY(gf_read_q(fs->quantized, &qcodes, &qscales, &qzps, &qn, &qd));
        hold.keep(qcodes);
        hold.keep(qscales);
        hold.keep(qzps);
        if (qn != n || qd != dim) return fail(GF_ERR_FORMAT, ".q file does not match the data file");
    }
    int32_t* attrs_i;
    uint32_t an, aa;
    TRY(gf_read_attrs(fs->attrs, &attrs_i, &an, &aa));
    hold.keep(attrs_i);
    uint32_t gn, ga, *grid, *cell_of;
    int32_t *lq, *rq;
    std::vector<uint32_t> ugrid, ucell;
    std::vector<int32_t> ulq, urq;
    if (fs->grid && fs->grid[0]) {
        TRY(gf_read_grid(fs->grid, &gn, &ga, &grid, &lq, &rq, &cell_of));
        hold.keep(grid);
        hold.keep(lq);
        hold.keep(rq);
        hold.keep(cell_of);
    } else {
        // uniform grid: slices of equal width over [lo, hi), cells by attribute value
        if (!fs->uniform_shape || fs->uniform_dims != aa || !(fs->uniform_hi > fs->uniform_lo))
            return fail(GF_ERR_ARG, "no grid file and no uniform grid matching the attribute count");
        gn = an;
        ga = aa;
        ugrid.assign(fs->uniform_shape, fs->uniform_shape + ga);
        for (uint32_t j = 0; j < ga; ++j) {
            if (ugrid[j] == 0) return fail(GF_ERR_ARG, "zero uniform grid size");
            const double w = ((double)fs->uniform_hi - fs->uniform_lo) / ugrid[j];
            for (uint32_t sl = 0; sl < ugrid[j]; ++sl) {
                ulq.push_back((int32_t)std::ceil(fs->uniform_lo + sl * w));
                urq.push_back((int32_t)std::ceil(fs->uniform_lo + (sl + 1) * w) - 1);
            }
        }
        ucell.resize(an);
        for (uint32_t i = 0; i < an; ++i) {
            uint32_t cell = 0;
            for (uint32_t j = 0; j < ga; ++j) {
                const double w = ((double)fs->uniform_hi - fs->uniform_lo) / ugrid[j];
                double sl = std::floor((attrs_i[(size_t)i * aa + j] - (double)fs->uniform_lo) / w);
                sl = std::min(std::max(sl, 0.0), (double)(ugrid[j] - 1));
                cell = cell * ugrid[j] + (uint32_t)sl;
            }
            ucell[i] = cell;
        }
        grid = ugrid.data();
        lq = ulq.data();
        rq = urq.data();
        cell_of = ucell.data();
    }
    if (gn != n) return fail(GF_ERR_FORMAT, "grid point count differs from the data file");
    if (an != n || aa != ga) return fail(GF_ERR_FORMAT, "attrs shape differs from data/grid");
    uint32_t ncells = 1, nq = 0;
    for (uint32_t j = 0; j < ga; ++j) {
        ncells *= grid[j];
        nq += grid[j];
    }
    std::vector<uint32_t> sizes(ncells, 0);
    for (uint32_t i = 0; i < n; ++i) {
        if (cell_of[i] >= ncells) return fail(GF_ERR_FORMAT, "grid cell id out of range");
        sizes[cell_of[i]]++;
    }
    // per-cell graphs, concatenated in cell order (check.cu:406-484)
    std::vector<uint32_t> graphs((size_t)n * fs->degree);
    size_t row = 0;
    for (uint32_t c = 0; c < ncells; ++c) {
        std::string p = std::string(fs->cagra_prefix ? fs->cagra_prefix : "") + std::to_string(c) +
                        (fs->cagra_suffix ? fs->cagra_suffix : "");
        uint32_t *gdat, gnum, gdeg;
        TRY(gf_read_u32mat(p.c_str(), &gdat, &gnum, &gdeg));
        hold.keep(gdat);
        if (gnum != sizes[c]) return fail(GF_ERR_FORMAT, "graph " + p + " row count differs from its cell size");
        if (gdeg != fs->degree) return fail(GF_ERR_FORMAT, "graph " + p + " degree differs from --degree");
        std::memcpy(&graphs[row * fs->degree], gdat, 4ull * gnum * gdeg);
        row += gnum;
    }
    uint32_t *cross = nullptr, cn = 0, ck = 0;
    TRY(gf_read_u32mat(fs->global_graph, &cross, &cn, &ck));
    hold.keep(cross);
    if (cn != n || ck % ncells != 0) return fail(GF_ERR_FORMAT, "global graph shape differs from n x cells*E");
    int32_t* labels = nullptr;
    uint32_t ln = 0;
    if (fs->cluster && fs->cluster[0]) {
        TRY(gf_read_labels(fs->cluster, &labels, &ln));
        hold.keep(labels);
        if (ln != n) return fail(GF_ERR_FORMAT, "cluster label count differs from the data file");
    }
    std::vector<float> attrs((size_t)n * ga), lqf(nq), rqf(nq);
    for (size_t i = 0; i < attrs.size(); ++i) attrs[i] = (float)attrs_i[i];  // realdataset_search.cu:2185-2190
    for (uint32_t i = 0; i < nq; ++i) {
        lqf[i] = (float)lq[i];  // real_dataset_adapter.cuh:604-609
        rqf[i] = (float)rq[i];
    }
    gf_index_desc d;
    std::memset(&d, 0, sizeof(d));
    d.n = n;
    d.dim = dim;
    d.n_attr = ga;
    d.vectors = vec;
    d.attrs = attrs.data();
    d.grid = grid;
    d.l_quant = lqf.data();
    d.r_quant = rqf.data();
    d.cell_of = cell_of;
    d.degree = fs->degree;
    d.graphs = graphs.data();
    d.cross_e = ck / ncells;
    d.cross = cross;
    d.n_clusters = labels ? 1 : 0;
    d.labels = labels;
    d.f2h_factor = fs->f2h_factor;
    d.keep_fp32 = fs->keep_fp32;
    d.host_graph = fs->host_graph;
    d.codec = fs->codec;
    if (fs->codec == 1 && qcodes) {
        d.codes = reinterpret_cast<const uint8_t*>(qcodes);
        d.code_scales = qscales;
        d.code_zero_points = qzps;
    } else if (fs->codec == 2) {
        d.codes = u8;
    }
    return gf_index_create(&d, device, out);
}

}  // extern "C"
