// Byte codecs of the stored vectors (row a18): per-dimension affine int8 and uint8.
//
// int8 quantisation restates the reference's host quantiser
// (load_dataset_return_int8_arr_infile, production_adapter.cuh:316-337; the same formula
// as the device kernel integer_production_kernal, :8-47, which rounds half to even where the
// host code rounds half away from zero; the host rule is used here, on both sides):
//   x = data * alpha; per dimension min / max over all points, starting from
//   min = 100000, max = -100000; scale = (max - min) / 255; zero_point = round(-128 -
//   min / scale) clamped to [-128, 127]; q = round(x / scale) + zero_point clamped to
//   [-128, 127]; round = half away from zero.  A dimension with max == min gets scale 1
//   (the reference divides by zero there).
// Decoding (big_dataset_adapterV3.cuh:852-863) is scale * (q - zero_point).  uint8 rows
// (the u8bin datasets, big_dataset_adapterV3.cuh:2802-2810, which decode byte / 100) use
// the same form with zero_point 0 and scale 0.01 by default.
#include <algorithm>
#include <cmath>
#include <cstring>

#include "gf_internal.h"

namespace gf {
namespace {

// Order-preserving map of floats to unsigned ints (for atomic min / max).
__device__ __forceinline__ uint32_t f2ord(float f) {
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float ord2f(uint32_t u) {
    return __uint_as_float((u & 0x80000000u) ? (u & 0x7FFFFFFFu) : ~u);
}
uint32_t f2ord_host(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Per-dimension min / max of data * alpha; 32 columns x 8 row lanes per block.
__global__ void minmax_kernel(const float* __restrict__ data, uint32_t n, uint32_t dim, float alpha,
                              uint32_t* __restrict__ mn, uint32_t* __restrict__ mx) {
    __shared__ float smin[8][33], smax[8][33];
    const uint32_t col = blockIdx.x * 32 + threadIdx.x;
    float lo = 100000.0f, hi = -100000.0f;
    if (col < dim)
        for (size_t r = (size_t)blockIdx.y * 8 + threadIdx.y; r < n; r += (size_t)gridDim.y * 8) {
            const float x = __fmul_rn(data[r * dim + col], alpha);
            lo = fminf(lo, x);
            hi = fmaxf(hi, x);
        }
    smin[threadIdx.y][threadIdx.x] = lo;
    smax[threadIdx.y][threadIdx.x] = hi;
    __syncthreads();
    if (threadIdx.y == 0 && col < dim) {
        for (int y = 1; y < 8; ++y) {
            lo = fminf(lo, smin[y][threadIdx.x]);
            hi = fmaxf(hi, smax[y][threadIdx.x]);
        }
        atomicMin(mn + col, f2ord(lo));
        atomicMax(mx + col, f2ord(hi));
    }
}

__global__ void params_kernel(const uint32_t* __restrict__ mn, const uint32_t* __restrict__ mx, uint32_t dim,
                              float* __restrict__ scales, int32_t* __restrict__ zps) {
    const uint32_t j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= dim) return;
    const float lo = ord2f(mn[j]), hi = ord2f(mx[j]);
    float scale = __fdiv_rn(__fsub_rn(hi, lo), 255.0f);
    if (!(scale > 0.0f)) scale = 1.0f;
    int zp = (int)roundf(__fsub_rn(-128.0f, __fdiv_rn(lo, scale)));
    scales[j] = scale;
    zps[j] = min(127, max(-128, zp));
}

__global__ void quantize_kernel(const float* __restrict__ data, size_t total, uint32_t dim, float alpha,
                                const float* __restrict__ scales, const int32_t* __restrict__ zps,
                                int8_t* __restrict__ q) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const uint32_t j = (uint32_t)(i % dim);
        const float x = __fmul_rn(data[i], alpha);
        const int v = (int)roundf(__fdiv_rn(x, scales[j])) + zps[j];
        q[i] = (int8_t)min(127, max(-128, v));
    }
}

}  // namespace

void quantize_i8_host(const float* data, uint32_t n, uint32_t dim, float alpha, int8_t* q, float* scales,
                      int32_t* zps) {
    std::vector<float> lo(dim, 100000.0f), hi(dim, -100000.0f);
    for (size_t i = 0; i < n; ++i)
        for (uint32_t j = 0; j < dim; ++j) {
            const float x = data[i * dim + j] * alpha;
            lo[j] = std::fmin(lo[j], x);
            hi[j] = std::fmax(hi[j], x);
        }
    for (uint32_t j = 0; j < dim; ++j) {
        float scale = (hi[j] - lo[j]) / 255.0f;
        if (!(scale > 0.0f)) scale = 1.0f;
        const int zp = (int)std::round(-128.0f - lo[j] / scale);
        scales[j] = scale;
        zps[j] = std::min(127, std::max(-128, zp));
    }
    if (!q) return;
    for (size_t i = 0; i < n; ++i)
        for (uint32_t j = 0; j < dim; ++j) {
            const float x = data[i * dim + j] * alpha;
            const int v = (int)std::round(x / scales[j]) + zps[j];
            q[i * dim + j] = (int8_t)std::min(127, std::max(-128, v));
        }
}

}  // namespace gf

using namespace gf;

extern "C" gf_status gf_quantize_i8_host(const float* data, uint32_t n, uint32_t dim, float alpha, int8_t* q_out,
                                         float* scales_out, int32_t* zero_points_out) {
    if ((!data && n) || !scales_out || !zero_points_out || dim == 0) return fail(GF_ERR_ARG, "null argument");
    quantize_i8_host(data, n, dim, alpha, q_out, scales_out, zero_points_out);
    return GF_OK;
}

extern "C" gf_status gf_quantize_i8(const float* data, uint32_t n, uint32_t dim, float alpha, int8_t* q_out,
                                    float* scales_out, int32_t* zero_points_out, void* stream) {
    if ((!data && n) || !q_out || !scales_out || !zero_points_out || dim == 0)
        return fail(GF_ERR_ARG, "null argument");
    cudaStream_t s = (cudaStream_t)stream;
    uint32_t* mm = nullptr;
    GF_CUDA(cudaMallocAsync((void**)&mm, sizeof(uint32_t) * 2 * dim, s));
    std::vector<uint32_t> init(2 * dim);
    for (uint32_t j = 0; j < dim; ++j) {
        init[j] = f2ord_host(100000.0f);
        init[dim + j] = f2ord_host(-100000.0f);
    }
    gf_status st = GF_OK;
    cudaError_t e = cudaMemcpyAsync(mm, init.data(), init.size() * 4, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) {
        dim3 grid((dim + 31) / 32, std::max<uint32_t>(1, std::min<uint32_t>((n + 255) / 256, 1024)));
        minmax_kernel<<<grid, dim3(32, 8), 0, s>>>(data, n, dim, alpha, mm, mm + dim);
        params_kernel<<<(dim + 127) / 128, 128, 0, s>>>(mm, mm + dim, dim, scales_out, zero_points_out);
        const size_t total = (size_t)n * dim;
        if (total)
            quantize_kernel<<<(unsigned)std::min<size_t>((total + 255) / 256, 148 * 32), 256, 0, s>>>(
                data, total, dim, alpha, scales_out, zero_points_out, q_out);
        e = cudaGetLastError();
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);  // init must outlive the copy
    }
    if (e != cudaSuccess) st = cuda_fail(e, "gf_quantize_i8");
    cudaFreeAsync(mm, s);
    return st;
}
