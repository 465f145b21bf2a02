// Test infrastructure: runs the reference's spokesman compression of the cross-cell graph,
// compress_global_graph_extreme (tools.cuh:917-1010), and its file writer
// save_global_graph_extreme (tools.cuh:1012-1038), compiled from the reference's own
// tools.cuh, on the CPU.  Both are host loops whose only device calls allocate buffers and
// copy the rank array; this driver maps cudaMallocHost / cudaMalloc / cudaMemcpy to host
// allocation and memcpy at compile time, so the reference's code runs unchanged without a
// GPU.  Built by oracle/Makefile (target ref_spokesman) into oracle/_ref/; never linked
// into the product.
//
//   ref_spokesman graphs.u32 sizes.u32 cross_t.u32 degree E out.bin
//     graphs.u32  concatenated per-cell graphs (local ids), rows in cell order
//     sizes.u32   points per cell
//     cross_t.u32 cross edges transposed: [cell][position][E] local ids
//     out.bin     the reference's compressed-graph file
#include <cuda_runtime.h>

#include <cstdlib>
#include <cstring>

static cudaError_t host_alloc_(void** p, size_t n) {
    *p = malloc(n ? n : 1);
    return *p ? cudaSuccess : cudaErrorMemoryAllocation;
}
#define cudaMallocHost(p, n) host_alloc_((void**)(p), (n))
#define cudaMalloc(p, n) host_alloc_((void**)(p), (n))
#define cudaMemcpy(d, s, n, k) (memcpy((d), (s), (n)), cudaSuccess)

#include "tools.cuh"

#include <cstdio>
#include <vector>

static std::vector<unsigned> read_all(const char* path) {
    std::vector<unsigned> v;
    FILE* f = fopen(path, "rb");
    if (!f) return v;
    fseek(f, 0, SEEK_END);
    long sz = ftell(f);
    fseek(f, 0, SEEK_SET);
    v.resize(sz / 4);
    if (fread(v.data(), 4, v.size(), f) != v.size()) v.clear();
    fclose(f);
    return v;
}

int main(int argc, char** argv) {
    if (argc != 7) return 2;
    std::vector<unsigned> graphs = read_all(argv[1]), sizes = read_all(argv[2]), cross_t = read_all(argv[3]);
    const unsigned degree = (unsigned)atoi(argv[4]), E = (unsigned)atoi(argv[5]);
    const unsigned pnum = (unsigned)sizes.size();
    unsigned n = 0;
    std::vector<unsigned> start(pnum), gstart(pnum);
    for (unsigned c = 0; c < pnum; ++c) {
        start[c] = n;
        gstart[c] = n * degree;
        n += sizes[c];
    }
    if (graphs.size() != (size_t)n * degree || cross_t.size() != (size_t)pnum * n * E) return 3;
    std::array<unsigned*, 3> graph_infos = {graphs.data(), sizes.data(), gstart.data()};
    std::array<unsigned*, 5> g = compress_global_graph_extreme(graph_infos, degree, cross_t.data(), pnum, n, E,
                                                               start.data());
    save_global_graph_extreme(std::string(argv[6]), g, pnum, n, E);
    return 0;
}
