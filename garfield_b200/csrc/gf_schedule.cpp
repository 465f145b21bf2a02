// Cell-batch scheduler for gf_search_batched.
//
// The reference's out-of-core driver processes a fixed random partition of the cells
// into batches (bigdataset_experiment.cu:271-277), although its README (README.md:5)
// describes choosing batches to minimise the queries that are active in many batches.
// A query whose cells fall into b different batches is searched b times from fresh
// entry points and loses the candidate reuse of cross-cell hops between those batches,
// so the quantity to minimise is the number of (query, batch) pairs, "splits".
//
// Greedy grouping by co-occurrence: w[c] = queries visiting cell c, M[c][c'] = queries
// visiting both.  Each batch starts from the unscheduled cell of largest w and repeatedly
// adds the unscheduled cell with the largest sum of M towards the batch's cells (ties:
// larger w, then smaller id) until it holds max_cells cells.  Cells that no query visits
// are not scheduled (nothing needs to be copied for them).
#include <algorithm>
#include <cstring>
#include <vector>

#include "gf_internal.h"

using namespace gf;

extern "C" gf_status gf_schedule_batches_host(uint32_t ncells, uint32_t qnum, const uint32_t* counts,
                                              const uint32_t* offsets, const uint32_t* cells, uint32_t max_cells,
                                              uint32_t* batch_cells_out, uint32_t* batch_sizes_out,
                                              uint32_t* n_batches_out, uint64_t* splits_out) {
    if (max_cells == 0) return fail(GF_ERR_ARG, "max_cells must be > 0");
    if (!batch_cells_out || !batch_sizes_out || !n_batches_out) return fail(GF_ERR_ARG, "null output");
    if (qnum && (!counts || !offsets || !cells)) return fail(GF_ERR_ARG, "null plan arrays");
    if (ncells > 65536) return fail(GF_ERR_ARG, "more than 65536 cells");
    const size_t P = ncells;
    std::vector<uint32_t> w(P, 0);
    std::vector<uint32_t> M(P * P, 0);
    for (uint32_t q = 0; q < qnum; ++q) {
        const uint32_t* cl = cells + offsets[q];
        for (uint32_t i = 0; i < counts[q]; ++i) {
            if (cl[i] >= ncells) return fail(GF_ERR_ARG, "plan cell id out of range");
            ++w[cl[i]];
            for (uint32_t j = 0; j < counts[q]; ++j)
                if (j != i) ++M[(size_t)cl[i] * P + cl[j]];
        }
    }
    std::vector<uint8_t> done(P, 0);
    std::vector<uint32_t> batch_of(P, kEmpty);
    std::vector<uint64_t> gain(P, 0);
    uint32_t nb = 0, filled = 0;
    for (;;) {
        uint32_t seed = kEmpty;
        for (uint32_t c = 0; c < ncells; ++c)
            if (!done[c] && w[c] > 0 && (seed == kEmpty || w[c] > w[seed])) seed = c;
        if (seed == kEmpty) break;
        std::fill(gain.begin(), gain.end(), 0);
        uint32_t size = 0;
        for (uint32_t add = seed; add != kEmpty;) {
            done[add] = 1;
            batch_of[add] = nb;
            batch_cells_out[filled++] = add;
            ++size;
            for (uint32_t c = 0; c < ncells; ++c) gain[c] += M[(size_t)add * P + c];
            add = kEmpty;
            if (size == max_cells) break;
            for (uint32_t c = 0; c < ncells; ++c) {
                if (done[c] || w[c] == 0) continue;
                if (add == kEmpty || gain[c] > gain[add] || (gain[c] == gain[add] && w[c] > w[add])) add = c;
            }
        }
        batch_sizes_out[nb++] = size;
    }
    *n_batches_out = nb;
    if (splits_out) {
        uint64_t splits = 0;
        std::vector<uint32_t> seen(nb ? nb : 1, kEmpty);
        for (uint32_t q = 0; q < qnum; ++q)
            for (uint32_t i = 0; i < counts[q]; ++i) {
                const uint32_t b = batch_of[cells[offsets[q] + i]];
                if (seen[b] != q) {
                    seen[b] = q;
                    ++splits;
                }
            }
        *splits_out = splits;
    }
    return GF_OK;
}

extern "C" gf_status gf_schedule_batches(gf_plan* plan, uint32_t max_cells, uint32_t* batch_cells_out,
                                         uint32_t* batch_sizes_out, uint32_t* n_batches_out, uint64_t* splits_out) {
    if (!plan) return fail(GF_ERR_ARG, "null plan");
    Plan& p = plan->p;
    if (!p.planned) return fail(GF_ERR_STATE, "plan not built");
    const uint32_t q = p.qnum, P = p.idx->d.ncells;
    std::vector<uint32_t> counts(q), offsets(q), cells((size_t)q * P);
    gf_status st = gf_plan_read(plan, counts.data(), offsets.data(), cells.data(), cells.size(), nullptr, nullptr);
    if (st != GF_OK) return st;
    return gf_schedule_batches_host(P, q, counts.data(), offsets.data(), cells.data(), max_cells, batch_cells_out,
                                    batch_sizes_out, n_batches_out, splits_out);
}
