// gf_search_noalloc: plan + search of a query batch that allocates no memory.
//
// Some callers cannot allocate device memory at query time: a serving thread with a
// latency budget cannot absorb a cudaMalloc (it can synchronise the device and take
// milliseconds), a process whose device memory has been claimed up front by another
// allocator has none left to hand out, and embedded callers under a fixed memory budget
// may forbid allocations after start-up.  For them this entry point keeps all of its
// working memory (the planned cell lists, the query copies, the sort/scan temporaries and
// the counters the search kernel needs besides its inputs and outputs) in one
// file-scope __device__ array of kNoAllocScratchBytes.  Every GPU that loads the library
// holds that array until the process exits.
//
// The array's name in host code is a host-side stand-in, not a device address, so the
// first call on each device looks up the device address with cudaGetSymbolAddress (with
// that device current) and caches it; make that first call before any stream capture.
// All calls share the one array and it keeps the last call's contents: the counters that
// must start at zero are cleared on the stream by every call, and calls that overlap on
// the GPU (two streams, or two threads) race on the array.
#include <cub/cub.cuh>

#include <mutex>

#include "gf_internal.h"

namespace gf {
namespace {

constexpr size_t kNoAllocScratchBytes = 4u << 20;  // 4 MiB per device
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
unsigned char* g_addr[kMaxDevices] = {nullptr};

// Device address of the scratch array on the current device (looked up once per device).
gf_status scratch_address(int device, unsigned char** out) {
    if (device < 0 || device >= kMaxDevices) return fail(GF_ERR_ARG, "device ordinal out of range");
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_addr[device]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress (no-allocation scratch)");
        g_addr[device] = static_cast<unsigned char*>(p);
    }
    *out = g_addr[device];
    return GF_OK;
}

struct Carver {
    unsigned char* base;
    size_t used = 0;
    template <typename T>
    T* take(size_t count) {
        size_t off = (used + 255) & ~size_t(255);
        used = off + std::max<size_t>(count, 1) * sizeof(T);
        return reinterpret_cast<T*>(base + off);
    }
};

struct DeviceGuard3 {
    int prev = -1;
    explicit DeviceGuard3(int d) {
        cudaGetDevice(&prev);
        cudaSetDevice(d);
    }
    ~DeviceGuard3() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

}  // namespace
}  // namespace gf

using namespace gf;

extern "C" gf_status gf_search_noalloc(gf_index* idx, const float* queries, const float* lb, const float* rb,
                                       uint32_t qnum, float prefilter, const gf_search_params* params,
                                       uint32_t* ids_out, float* dist_out, void* stream) {
    if (!idx) return fail(GF_ERR_ARG, "null index");
    if (qnum == 0) return GF_OK;
    if (!queries || !lb || !rb || !ids_out) return fail(GF_ERR_ARG, "null argument");
    DeviceIndex& d = idx->d;
    if (d.sharded || d.host_graph) return fail(GF_ERR_STATE, "gf_search_noalloc needs a whole device-resident index");
    if (params && params->exact_tc)
        return fail(GF_ERR_ARG, "exact_tc needs the tensor-core pass's working memory (use gf_search)");
    DeviceGuard3 guard(d.device);
    unsigned char* scratch = nullptr;
    gf_status st = scratch_address(d.device, &scratch);
    if (st != GF_OK) return st;

    // Lay the plan's buffers out inside the scratch array (sizes as gf_plan_create).
    gf_plan plan;
    Plan& p = plan.p;
    p.idx = idx;
    p.device = d.device;
    p.max_q = qnum;
    Carver cv{scratch};
    const size_t Q = qnum;
    p.q16 = cv.take<uint4>(Q * d.d8 / 8);
    p.q32 = cv.take<float>(Q * d.dim);
    p.lb = cv.take<float>(Q * d.a);
    p.rb = cv.take<float>(Q * d.a);
    p.counts = cv.take<uint32_t>(Q);
    p.offsets = cv.take<uint32_t>(Q);
    p.cells = cv.take<uint32_t>(Q * d.ncells);
    p.top4 = cv.take<uint32_t>(Q * 4);
    p.part_d = cv.take<float>(Q * centroid_splits(d.C) * 4);
    p.part_i = cv.take<uint32_t>(Q * centroid_splits(d.C) * 4);
    p.box = cv.take<uint32_t>(Q);
    p.task = cv.take<uint32_t>(Q * 3);
    p.scratch = cv.take<uint32_t>(16);
    p.stats = cv.take<unsigned long long>(8);
    size_t t1 = 0, t2 = 0;
    cub::DeviceScan::ExclusiveSum(nullptr, t1, p.counts, p.offsets, (int)Q);
    cub::DeviceRadixSort::SortPairsDescending(nullptr, t2, p.counts, p.task, p.task, p.task, (int)Q, 0,
                                              count_sort_bits(d.ncells));
    p.scan_tmp_bytes = std::max(t1, t2);
    p.scan_tmp = cv.take<unsigned char>(p.scan_tmp_bytes);
    if (cv.used > kNoAllocScratchBytes)
        return fail(GF_ERR_ARG, "batch of " + std::to_string(qnum) + " queries needs " + std::to_string(cv.used) +
                                    " bytes of working memory; gf_search_noalloc has " +
                                    std::to_string(kNoAllocScratchBytes) + " (split the batch)");
    if (d.ncells > 1024) return fail(GF_ERR_ARG, "more than 1024 cells per index are not supported");

    cudaStream_t s = (cudaStream_t)stream;
    st = plan_queries(idx, &plan, queries, lb, rb, qnum, prefilter, s);
    if (st != GF_OK) return st;
    return gf::search(idx, &plan, params, ids_out, dist_out, s);
}
