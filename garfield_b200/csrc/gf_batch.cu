// Search over batches of cells: the out-of-core driver of the reference
// (batch_graph_search_gpu_with_prefilter_batch_process_compressed_graph_T_dataset_resident,
// big_dataset_adapterV3.cuh:3321-3715) re-designed around one search kernel with a cell view.
//
// Per batch b (turn t = b mod 2):
//   host: fill the batch's tables (slot of each cell, graph offset of each slot, cross
//         offset of each (target, source) slot pair) into pinned staging of turn t;
//   copy stream: after the search of batch b-2 (which used turn t's buffers) has finished
//         (stream event), copy the tables and, for an index with host_graph, the graph rows
//         of the batch's cells and the cross-edge blocks between them into turn t's device
//         buffers; record "copied[t]";
//   caller's stream: wait for copied[t] (stream event, no host synchronisation), run the
//         search kernel restricted to the batch, merging each query's k best into its
//         running keys; record "searched[t]".
// So the copies of batch b+1 overlap the search of batch b.  The reference instead copies
// on a non-blocking stream but synchronises the device per batch (:3603-3612) and merges
// each batch's list on 9 host threads (:3343-3395); here the merge is part of the kernel.
#include <algorithm>
#include <cstring>
#include <vector>

#include "gf_internal.h"

#define GF_TRY_STATUS(x)               \
    do {                               \
        gf_status s_ = (x);            \
        if (s_ != GF_OK) return s_;    \
    } while (0)

namespace gf {

struct BatchState {
    int device = -1;
    cudaStream_t copy = nullptr;
    cudaEvent_t copied[2] = {nullptr, nullptr};
    cudaEvent_t searched[2] = {nullptr, nullptr};
    bool used[2] = {false, false};
    unsigned char* tab_h[2] = {nullptr, nullptr};  // pinned table staging
    unsigned char* tab_d[2] = {nullptr, nullptr};
    size_t tab_bytes = 0;
    uint32_t* gbuf[2] = {nullptr, nullptr};  // streamed graph rows
    size_t gcap[2] = {0, 0};
    uint32_t* xbuf[2] = {nullptr, nullptr};  // streamed cross blocks
    size_t xcap[2] = {0, 0};
    unsigned long long* run = nullptr;  // qnum x k running keys
    size_t run_cap = 0;
};

void free_batch_state(BatchState* b) {
    if (!b) return;
    if (b->copy) cudaStreamSynchronize(b->copy);
    for (int t = 0; t < 2; ++t) {
        if (b->searched[t]) cudaEventSynchronize(b->searched[t]);
        if (b->copied[t]) cudaEventDestroy(b->copied[t]);
        if (b->searched[t]) cudaEventDestroy(b->searched[t]);
        if (b->tab_h[t]) cudaFreeHost(b->tab_h[t]);
        if (b->tab_d[t]) cudaFree(b->tab_d[t]);
        if (b->gbuf[t]) cudaFree(b->gbuf[t]);
        if (b->xbuf[t]) cudaFree(b->xbuf[t]);
    }
    if (b->run) cudaFree(b->run);
    if (b->copy) cudaStreamDestroy(b->copy);
    delete b;
}

namespace {

// Grow a device buffer of turn t to `words`, after the work that may still read it.
gf_status grow(uint32_t** buf, size_t* cap, size_t words, cudaEvent_t busy, bool used) {
    if (words <= *cap) return GF_OK;
    if (used) GF_CUDA(cudaEventSynchronize(busy));
    if (*buf) cudaFree(*buf);
    *buf = nullptr;
    *cap = 0;
    GF_CUDA(cudaMalloc((void**)buf, words * 4));
    *cap = words;
    return GF_OK;
}

}  // namespace

gf_status search_batched(gf_index* idx, gf_plan* plan, const gf_search_params* prm, const uint32_t* batch_cells,
                         const uint32_t* batch_sizes, uint32_t n_batches, uint32_t* ids, float* dist,
                         cudaStream_t s) {
    DeviceIndex& d = idx->d;
    Plan& p = plan->p;
    if (!p.planned) return fail(GF_ERR_STATE, "gf_search_batched before gf_plan_queries");
    if (d.sharded) return fail(GF_ERR_STATE, "gf_search_batched on a shard: search it with gf_search_keys");
    gf_search_params P;
    if (prm && prm->exact_tc) return fail(GF_ERR_ARG, "exact_tc applies to gf_search and gf_search_host");
    gf_search_defaults(&P);
    if (prm) P = *prm;
    if (P.k == 0 || P.k > 1024) return fail(GF_ERR_ARG, "k must be 1..1024");
    if (!ids) return fail(GF_ERR_ARG, "null ids_out");
    if (n_batches && (!batch_cells || !batch_sizes)) return fail(GF_ERR_ARG, "null batch arrays");
    const uint32_t NC = d.ncells, R = d.degree, E = d.E;
    // every cell in at most one batch
    std::vector<uint32_t> batch_of(NC, kEmpty);
    size_t total = 0, max_b = 0;
    for (uint32_t b = 0; b < n_batches; ++b) {
        for (uint32_t i = 0; i < batch_sizes[b]; ++i) {
            const uint32_t c = batch_cells[total + i];
            if (c >= NC) return fail(GF_ERR_ARG, "batch cell id out of range");
            if (batch_of[c] != kEmpty) return fail(GF_ERR_ARG, "cell " + std::to_string(c) + " in two batches");
            batch_of[c] = b;
        }
        total += batch_sizes[b];
        max_b = std::max<size_t>(max_b, batch_sizes[b]);
    }
    if (!p.batch) {
        p.batch = new BatchState();
        p.batch->device = d.device;
        GF_CUDA(cudaStreamCreateWithFlags(&p.batch->copy, cudaStreamNonBlocking));
        for (int t = 0; t < 2; ++t) {
            GF_CUDA(cudaEventCreateWithFlags(&p.batch->copied[t], cudaEventDisableTiming));
            GF_CUDA(cudaEventCreateWithFlags(&p.batch->searched[t], cudaEventDisableTiming));
        }
    }
    BatchState& bs = *p.batch;
    // table block: slot (NC int32, padded to 8 bytes) | gofs (B int64) | xofs (B*B int64)
    const size_t slot_bytes = ((size_t)NC * 4 + 7) & ~size_t(7);
    const size_t tab_need = slot_bytes + 8 * (max_b + max_b * max_b);
    if (tab_need > bs.tab_bytes) {
        for (int t = 0; t < 2; ++t) {
            if (bs.used[t]) {
                GF_CUDA(cudaEventSynchronize(bs.copied[t]));
                GF_CUDA(cudaEventSynchronize(bs.searched[t]));
            }
            if (bs.tab_h[t]) cudaFreeHost(bs.tab_h[t]);
            if (bs.tab_d[t]) cudaFree(bs.tab_d[t]);
            bs.tab_h[t] = bs.tab_d[t] = nullptr;
        }
        bs.tab_bytes = 0;
        for (int t = 0; t < 2; ++t) {
            GF_CUDA(cudaMallocHost((void**)&bs.tab_h[t], tab_need));
            GF_CUDA(cudaMalloc((void**)&bs.tab_d[t], tab_need));
        }
        bs.tab_bytes = tab_need;
    }
    const size_t run_need = (size_t)p.qnum * P.k;
    if (run_need > bs.run_cap) {
        GF_CUDA(cudaStreamSynchronize(s));
        if (bs.run) cudaFree(bs.run);
        bs.run = nullptr;
        bs.run_cap = 0;
        GF_CUDA(cudaMalloc((void**)&bs.run, std::max<size_t>(run_need, 1) * 8));
        bs.run_cap = run_need;
    }
    GF_CUDA(cudaMemsetAsync(bs.run, 0xFF, run_need * 8, s));  // every key empty
    if (n_batches == 0) GF_CUDA(cudaMemsetAsync(p.stats, 0, 8 * sizeof(unsigned long long), s));

    size_t first = 0;
    for (uint32_t b = 0; b < n_batches; ++b) {
        const int t = b & 1;
        const uint32_t B = batch_sizes[b];
        const uint32_t* cb = batch_cells + first;
        first += B;
        // host staging of turn t was last read by the copies of batch b-2
        if (bs.used[t]) GF_CUDA(cudaEventSynchronize(bs.copied[t]));
        unsigned char* th = bs.tab_h[t];
        int32_t* slot = reinterpret_cast<int32_t*>(th);
        long long* gofs = reinterpret_cast<long long*>(th + slot_bytes);
        long long* xofs = gofs + B;
        for (uint32_t c = 0; c < NC; ++c) slot[c] = -1;
        for (uint32_t i = 0; i < B; ++i) slot[cb[i]] = (int32_t)i;
        CellView v;
        size_t pts = 0;  // points in the batch
        for (uint32_t i = 0; i < B; ++i) pts += d.seg_h[cb[i] + 1] - d.seg_h[cb[i]];
        // cross rows of a cell: its positions, or its spokesmen's ranks (compressed edges);
        // xofs entries are a block's start less its first row times the row stride
        const bool spkr = !d.spk_start_h.empty();
        auto row0 = [&](uint32_t c) -> size_t { return spkr ? d.spk_start_h[c] : d.seg_h[c]; };
        auto nrows = [&](uint32_t c) -> size_t {
            return spkr ? d.spk_start_h[c + 1] - d.spk_start_h[c] : d.seg_h[c + 1] - d.seg_h[c];
        };
        size_t xrows = 0;  // cross rows of the batch's cells
        for (uint32_t i = 0; i < B; ++i) xrows += nrows(cb[i]);
        if (!d.host_graph) {
            for (uint32_t i = 0; i < B; ++i) gofs[i] = (long long)d.seg_h[cb[i]] * R;
            for (uint32_t it = 0; it < B; ++it)
                for (uint32_t is = 0; is < B; ++is) xofs[(size_t)it * B + is] = (long long)cb[it] * E;
            v.graph = d.graph;
            v.cross = d.cross;
            v.xstride = NC * E;
        } else {
            long long g = 0;
            for (uint32_t i = 0; i < B; ++i) {
                gofs[i] = g;
                g += (long long)(d.seg_h[cb[i] + 1] - d.seg_h[cb[i]]) * R;
            }
            long long x = 0;
            for (uint32_t it = 0; it < B; ++it)
                for (uint32_t is = 0; is < B; ++is) {
                    xofs[(size_t)it * B + is] = x - (long long)row0(cb[is]) * E;
                    x += (long long)nrows(cb[is]) * E;
                }
            GF_TRY_STATUS(grow(&bs.gbuf[t], &bs.gcap[t], std::max<size_t>(pts * R, 1), bs.searched[t], bs.used[t]));
            GF_TRY_STATUS(
                grow(&bs.xbuf[t], &bs.xcap[t], std::max<size_t>(xrows * B * E, 1), bs.searched[t], bs.used[t]));
            v.graph = bs.gbuf[t];
            v.cross = bs.xbuf[t];
            v.xstride = E;
        }
        // copies of turn t wait for the search that last used turn t's device buffers
        if (bs.used[t]) GF_CUDA(cudaStreamWaitEvent(bs.copy, bs.searched[t], 0));
        const size_t tab_used = slot_bytes + 8 * ((size_t)B + (size_t)B * B);
        GF_CUDA(cudaMemcpyAsync(bs.tab_d[t], th, tab_used, cudaMemcpyHostToDevice, bs.copy));
        if (d.host_graph) {
            for (uint32_t i = 0; i < B; ++i) {
                const uint32_t c = cb[i];
                const size_t rows = d.seg_h[c + 1] - d.seg_h[c];
                if (rows)
                    GF_CUDA(cudaMemcpyAsync(bs.gbuf[t] + gofs[i], d.graph_h + (size_t)d.seg_h[c] * R, rows * R * 4,
                                            cudaMemcpyHostToDevice, bs.copy));
            }
            if (E)
                for (uint32_t it = 0; it < B; ++it)
                    for (uint32_t is = 0; is < B; ++is) {
                        const uint32_t ct = cb[it], cs = cb[is];
                        const size_t rows = nrows(cs);
                        if (rows)
                            GF_CUDA(cudaMemcpyAsync(bs.xbuf[t] + xofs[(size_t)it * B + is] + (long long)row0(cs) * E,
                                                    d.cross_h + ((size_t)ct * d.cross_rows + row0(cs)) * E,
                                                    rows * E * 4, cudaMemcpyHostToDevice, bs.copy));
                    }
        }
        GF_CUDA(cudaEventRecord(bs.copied[t], bs.copy));
        bs.used[t] = true;
        GF_CUDA(cudaStreamWaitEvent(s, bs.copied[t], 0));
        v.slot = reinterpret_cast<const int32_t*>(bs.tab_d[t]);
        v.gofs = reinterpret_cast<const long long*>(bs.tab_d[t] + slot_bytes);
        v.xofs = v.gofs + B;
        v.nslots = B;
        v.run = bs.run;
        v.accumulate_stats = b > 0;
        gf_status st = gf::search(idx, plan, &P, nullptr, nullptr, s, &v);
        if (st != GF_OK) return st;
        GF_CUDA(cudaEventRecord(bs.searched[t], s));
    }
    return finish_run(idx, bs.run, (uint32_t)run_need, ids, dist, s);
}

}  // namespace gf

using namespace gf;

extern "C" gf_status gf_search_batched(gf_index* idx, gf_plan* plan, const gf_search_params* params,
                                       const uint32_t* batch_cells, const uint32_t* batch_sizes, uint32_t n_batches,
                                       uint32_t* ids_out, float* dist_out, void* stream) {
    if (!idx || !plan || plan->p.idx != idx) return fail(GF_ERR_ARG, "plan does not belong to this index");
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(idx->d.device);
    gf_status st = search_batched(idx, plan, params, batch_cells, batch_sizes, n_batches, ids_out, dist_out,
                                  (cudaStream_t)stream);
    if (prev >= 0) cudaSetDevice(prev);
    return st;
}
