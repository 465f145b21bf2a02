// Exact filtered k-NN on the fp32 rows: the GPU ground truth.  Replaces
// naive_brute_force_with_filter (gpu_graph.cu:10782-10812, CPU, one query per OpenMP
// thread) and prefiltering_and_bruteforce (brute_force.cuh:331, fp16 distances).
// One 256-thread block per query: every point's attributes are tested (coalesced
// reads over the cell-major attribute array), in-range points are compacted per warp
// and their canonical fp32 distances computed thread-per-point; each warp keeps a
// sorted top-k list in shared memory, merged at the end.  Order: (distance, global id).
#include <algorithm>
#include <mutex>

#include "gf_device.cuh"
#include "gf_internal.h"

namespace gf {
namespace {

using namespace dev;

constexpr uint32_t kBfWarps = 8;

__global__ void __launch_bounds__(256) bruteforce_kernel(const float4* __restrict__ vec32, const float* __restrict__ attrs,
                                                         const uint32_t* __restrict__ i2g, uint32_t n, uint32_t nch,
                                                         uint32_t a, const float* __restrict__ queries, uint32_t dim,
                                                         const float* __restrict__ lb, const float* __restrict__ rb,
                                                         uint32_t k, uint32_t* __restrict__ ids,
                                                         float* __restrict__ dists, const uint32_t* __restrict__ qlist,
                                                         const uint32_t* __restrict__ qcount) {
    extern __shared__ __align__(16) float sm[];
    // with a query list, block b answers query qlist[b] (blocks past *qcount have none)
    if (qlist && blockIdx.x >= *qcount) return;
    const uint32_t q = qlist ? qlist[blockIdx.x] : blockIdx.x, lane = lane_id(), w = threadIdx.x >> 5;
    float4* qs = reinterpret_cast<float4*>(sm);                 // nch
    float* sl = sm + nch * 4;                                   // a
    float* sr = sl + kMaxAttr;                                  // a
    float* lists_d = sr + kMaxAttr;                             // kBfWarps x 2 x k (double buffer)
    uint32_t* lists_w = reinterpret_cast<uint32_t*>(lists_d + kBfWarps * 2 * k);
    float* bd_all = reinterpret_cast<float*>(lists_w + kBfWarps * 2 * k);  // kBfWarps x 32
    uint32_t* bw_all = reinterpret_cast<uint32_t*>(bd_all + kBfWarps * 32);

    for (uint32_t c = threadIdx.x; c < nch * 4; c += blockDim.x) {
        uint32_t d = c;
        reinterpret_cast<float*>(qs)[c] = d < dim ? queries[(size_t)q * dim + d] : 0.0f;
    }
    if (threadIdx.x < a) {
        sl[threadIdx.x] = lb[(size_t)q * a + threadIdx.x];
        sr[threadIdx.x] = rb[(size_t)q * a + threadIdx.x];
    }
    for (uint32_t i = threadIdx.x; i < kBfWarps * 2 * k; i += blockDim.x) {
        lists_d[i] = __int_as_float(0x7f800000);
        lists_w[i] = kEmpty;
    }
    __syncthreads();

    float* ld = lists_d + w * 2 * k;
    uint32_t* lw = lists_w + w * 2 * k;
    float* nd = ld + k;
    uint32_t* nw = lw + k;
    float* bd = bd_all + w * 32;
    uint32_t* bw = bw_all + w * 32;

    // each warp scans a contiguous slice of positions, 32 at a time
    const uint32_t per = (n + kBfWarps - 1) / kBfWarps;
    const uint32_t beg = w * per, end = min(n, beg + per);
    uint32_t nb = 0;
    for (uint32_t x0 = beg; x0 < end; x0 += 32) {
        uint32_t x = x0 + lane;
        bool ok = x < end && in_box(attrs, x, a, sl, sr);
        uint32_t msk = __ballot_sync(kFull, ok);
        uint32_t cnt = __popc(msk);
        // flush first if the 32-slot buffer would overflow
        if (nb + cnt > 32) {
            __syncwarp();
            float dd = __int_as_float(0x7f800000);
            uint32_t ww = kEmpty;
            if (lane < nb) {
                uint32_t pos = bw[lane];
                dd = dist32(vec32 + (size_t)pos * nch, qs, nch);
                ww = __ldg(i2g + pos);
            }
            bd[lane] = dd;
            bw[lane] = ww;
            __syncwarp();
            warp_sort(bd, bw, 32);
            if (lw[k - 1] == kEmpty || mkkey(bd[0], bw[0]) < mkkey(ld[k - 1], lw[k - 1])) {
                merge_list(ld, lw, nd, nw, k, bd, bw, nb, nullptr, nullptr, false);
                float* t = ld; ld = nd; nd = t;
                uint32_t* tw = lw; lw = nw; nw = tw;
            }
            nb = 0;
        }
        if (ok) bw[nb + __popc(msk & lanemask_lt())] = x;
        nb += cnt;
        __syncwarp();
    }
    if (nb) {
        float dd = __int_as_float(0x7f800000);
        uint32_t ww = kEmpty;
        if (lane < nb) {
            uint32_t pos = bw[lane];
            dd = dist32(vec32 + (size_t)pos * nch, qs, nch);
            ww = __ldg(i2g + pos);
        }
        __syncwarp();
        bd[lane] = dd;
        bw[lane] = ww;
        __syncwarp();
        warp_sort(bd, bw, 32);
        merge_list(ld, lw, nd, nw, k, bd, bw, nb, nullptr, nullptr, false);
        float* t = ld; ld = nd; nd = t;
        uint32_t* tw = lw; lw = nw; nw = tw;
    }
    // publish each warp's final list into its first buffer slot
    if (ld != lists_d + w * 2 * k) {
        for (uint32_t i = lane; i < k; i += 32) {
            lists_d[w * 2 * k + i] = ld[i];
            lists_w[w * 2 * k + i] = lw[i];
        }
    }
    __syncthreads();
    if (w == 0) {
        float* cd = lists_d;
        uint32_t* cw = lists_w;
        float* od = lists_d + k;
        uint32_t* ow = lists_w + k;
        for (uint32_t v = 1; v < kBfWarps; ++v) {
            float* vd = lists_d + v * 2 * k;
            uint32_t* vw = lists_w + v * 2 * k;
            uint32_t nv = 0;  // valid entries of warp v's list
            for (uint32_t i0 = 0; i0 < k; i0 += 32) {
                uint32_t i = i0 + lane;
                nv += __popc(__ballot_sync(kFull, i < k && vw[i] != kEmpty));
            }
            if (nv == 0) continue;
            merge_list(cd, cw, od, ow, k, vd, vw, nv, nullptr, nullptr, false);
            float* t = cd; cd = od; od = t;
            uint32_t* tw = cw; cw = ow; ow = tw;
        }
        for (uint32_t i = lane; i < k; i += 32) {
            ids[(size_t)q * k + i] = cw[i];
            if (dists) dists[(size_t)q * k + i] = cd[i];
        }
    }
}

}  // namespace

gf_status bruteforce(gf_index* idx, const float* queries, const float* lb, const float* rb, uint32_t qnum,
                     uint32_t k, uint32_t* ids, float* dist, cudaStream_t s, const gf_bf_params* prm,
                     const uint32_t* qmask) {
    DeviceIndex& d = idx->d;
    if (!d.vec32) return fail(GF_ERR_STATE, "index was created without keep_fp32");
    if (k == 0 || k > 1024) return fail(GF_ERR_ARG, "k must be 1..1024");
    gf_bf_params P{};
    if (prm) P = *prm;
    if (P.path > 2) return fail(GF_ERR_ARG, "path must be 0, 1 or 2");
    const bool tc = P.path != 1 && bf_tc_usable(d, k);
    if (qmask && !tc) return fail(GF_ERR_STATE, "a query mask needs the tensor-core pass");
    if (P.path == 2 && !tc)
        return fail(GF_ERR_ARG, "tensor-core brute force needs keep_fp32, dim <= 1024, finite rows and k <= 128");
    if (P.stats_out) GF_CUDA(cudaMemsetAsync(P.stats_out, 0, 3 * sizeof(uint32_t), s));
    if (qnum == 0) return GF_OK;
    if (!queries || !lb || !rb || !ids) return fail(GF_ERR_ARG, "null argument");
    const uint32_t nch = d.d4 / 4;
    size_t smem = sizeof(float) * (nch * 4 + 2 * kMaxAttr) + (sizeof(float) + 4) * kBfWarps * 2 * k +
                  (sizeof(float) + 4) * kBfWarps * 32;
    int max_optin = 0;
    cudaDeviceGetAttribute(&max_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, d.device);
    if (smem > (size_t)max_optin) return fail(GF_ERR_ARG, "k or dim too large for the brute-force kernel");
    GF_CUDA(cudaFuncSetAttribute(bruteforce_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    if (!tc) {
        bruteforce_kernel<<<qnum, 256, smem, s>>>(d.vec32, d.attrs, d.i2g, d.n, nch, d.a, queries, d.dim, lb, rb, k,
                                                  ids, dist, nullptr, nullptr);
        GF_CUDA(cudaGetLastError());
        return GF_OK;
    }
    // tensor-core pass, then the CUDA-core kernel for the queries it could not prove; working
    // memory: the pass's, then [0] fallback count, [1] timeouts, [2] tile products, [3..] list
    const size_t tc_bytes = (bf_tc_ws_bytes(d, qnum, k) + 255) & ~size_t(255);
    const size_t need = tc_bytes + sizeof(uint32_t) * (3 + (size_t)qnum);
    std::lock_guard<std::mutex> lock(*d.bf_mu);
    if (!d.bf_ws_ev) GF_CUDA(cudaEventCreateWithFlags(&d.bf_ws_ev, cudaEventDisableTiming));
    if (d.bf_ws_bytes < need) {
        GF_CUDA(cudaEventSynchronize(d.bf_ws_ev));  // the last call that used the buffer is done
        if (d.bf_ws) cudaFree(d.bf_ws);
        d.bf_ws = nullptr;
        d.bf_ws_bytes = 0;
        GF_CUDA(cudaMalloc(&d.bf_ws, need));
        d.bf_ws_bytes = need;
    }
    GF_CUDA(cudaStreamWaitEvent(s, d.bf_ws_ev, 0));  // calls on other streams that share the buffer
    uint32_t* w = reinterpret_cast<uint32_t*>(static_cast<unsigned char*>(d.bf_ws) + tc_bytes);
    gf_status st = GF_OK;
    cudaError_t e = cudaMemsetAsync(w, 0, 3 * sizeof(uint32_t), s);
    if (e != cudaSuccess) st = cuda_fail(e, "brute-force counters");
    if (st == GF_OK)
        st = bf_tc_run(idx, queries, lb, rb, qnum, k, ids, dist, d.bf_ws, w + 3, w, P.test_fallback_every, P.test_wait,
                       w + 1, w + 2, s, qmask);
    if (st == GF_OK) {
        bruteforce_kernel<<<qnum, 256, smem, s>>>(d.vec32, d.attrs, d.i2g, d.n, nch, d.a, queries, d.dim, lb, rb, k,
                                                  ids, dist, w + 3, w);
        e = cudaGetLastError();
        if (e == cudaSuccess && P.stats_out)
            e = cudaMemcpyAsync(P.stats_out, w, 3 * sizeof(uint32_t), cudaMemcpyDeviceToDevice, s);
        if (e != cudaSuccess) st = cuda_fail(e, "brute force");
    }
    const cudaError_t er = cudaEventRecord(d.bf_ws_ev, s);
    if (st == GF_OK && er != cudaSuccess) st = cuda_fail(er, "brute-force event");
    return st;
}

}  // namespace gf
