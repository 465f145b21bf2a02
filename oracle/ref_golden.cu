// Test infrastructure: a driver that runs host-side (CPU) functions of the
// reference's query path, compiled from the reference's own sources, to produce golden
// vectors for the oracle:
//   bf       naive_brute_force_with_filter (gpu_graph.cu:10782-10812), one call per query
//   bf_omp   the same scan over all queries under omp parallel for, timed (the CPU
//            baseline of bench.py --impl reference)
//   cluster  load_clustering (tools.cuh:569-602): centroids and the cell x cluster histogram
//   quant    load_dataset_return_int8_arr_infile (production_adapter.cuh:286-383): its host
//            quantiser writes the .q file before any device copy; without a GPU the device
//            copies that follow fail and are ignored by the reference's own error handling
// Built by oracle/Makefile (target ref_golden) into oracle/_ref/; never linked into the
// product.  Input/output files are plain little-endian arrays described below.
#include <unordered_map>
#include <unordered_set>

#include "gpu_graph.cu"
#include "production_adapter.cuh"

#include <chrono>
#include <cstdio>
#include <cstdlib>

static void write_u32(const char* path, const std::vector<unsigned>& v) {
    FILE* f = fopen(path, "wb");
    fwrite(v.data(), 4, v.size(), f);
    fclose(f);
}

int main(int argc, char** argv) {
    if (argc < 2) return 2;
    std::string mode = argv[1];
    if (mode == "bf" && argc == 8) {
        // bf data.fvecs attrs.bin queries.fvecs ranges.bin k out.u32
        unsigned num, dim, qnum, qdim, an, ad;
        float *data, *queries;
        int* attrs_i;
        load_data(std::string(argv[2]), data, num, dim);
        load_attrs<int>(std::string(argv[3]), attrs_i, ad, an);
        load_data(std::string(argv[4]), queries, qnum, qdim);
        std::vector<int> li(qnum * ad), ri(qnum * ad);
        load_range<int>(std::string(argv[5]), li.data(), ri.data(), ad, qnum);
        unsigned k = (unsigned)atoi(argv[6]);
        std::vector<float> attrs((size_t)an * ad), lf(li.begin(), li.end()), rf(ri.begin(), ri.end());
        for (size_t i = 0; i < attrs.size(); ++i) attrs[i] = (float)attrs_i[i];
        std::vector<unsigned> out((size_t)qnum * k, 0xFFFFFFFFu);
        for (unsigned q = 0; q < qnum; ++q) {
            std::vector<unsigned> r = naive_brute_force_with_filter(queries + (size_t)q * dim, data, dim, num, k,
                                                                    lf.data() + q * ad, rf.data() + q * ad,
                                                                    attrs.data(), ad);
            for (size_t j = 0; j < r.size() && j < k; ++j) out[(size_t)q * k + j] = r[j];
        }
        write_u32(argv[7], out);
        return 0;
    }
    if (mode == "bf_omp" && argc == 10) {
        // bf_omp data.fvecs attrs.bin queries.fvecs ranges.bin k threads chunk out.u32
        // The reference's own CPU scan timed the way its main calls it
        // (realdataset_search.cu:2330-2335: one call per query under omp parallel for),
        // with the given thread count, over consecutive chunks of `chunk` queries; prints
        // "seconds <wall time>" per chunk (file loading is not timed).
        unsigned num, dim, qnum, qdim, an, ad;
        float *data, *queries;
        int* attrs_i;
        load_data(std::string(argv[2]), data, num, dim);
        load_attrs<int>(std::string(argv[3]), attrs_i, ad, an);
        load_data(std::string(argv[4]), queries, qnum, qdim);
        std::vector<int> li(qnum * ad), ri(qnum * ad);
        load_range<int>(std::string(argv[5]), li.data(), ri.data(), ad, qnum);
        unsigned k = (unsigned)atoi(argv[6]);
        int threads = atoi(argv[7]);
        unsigned chunk = (unsigned)atoi(argv[8]);
        if (chunk == 0) chunk = qnum;
        std::vector<float> attrs((size_t)an * ad), lf(li.begin(), li.end()), rf(ri.begin(), ri.end());
        for (size_t i = 0; i < attrs.size(); ++i) attrs[i] = (float)attrs_i[i];
        std::vector<std::vector<unsigned>> res(qnum);
        for (unsigned c0 = 0; c0 < qnum; c0 += chunk) {
            unsigned c1 = std::min(qnum, c0 + chunk);
            auto t0 = std::chrono::steady_clock::now();
#pragma omp parallel for num_threads(threads)
            for (unsigned q = c0; q < c1; ++q)
                res[q] = naive_brute_force_with_filter(queries + (size_t)q * dim, data, dim, num, k,
                                                       lf.data() + q * ad, rf.data() + q * ad, attrs.data(), ad);
            double sec = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
            printf("seconds %.6f\n", sec);
        }
        std::vector<unsigned> out((size_t)qnum * k, 0xFFFFFFFFu);
        for (unsigned q = 0; q < qnum; ++q)
            for (size_t j = 0; j < res[q].size() && j < k; ++j) out[(size_t)q * k + j] = res[q][j];
        write_u32(argv[9], out);
        return 0;
    }
    if (mode == "cluster" && argc == 6) {
        // cluster data.fvecs cluster.bin centroids.f32 hist.u32
        unsigned num, dim;
        float* data;
        load_data(std::string(argv[2]), data, num, dim);
        std::vector<unsigned> cid;
        float* centers = nullptr;
        std::vector<std::vector<unsigned>> ncp;
        load_clustering(cid, std::string(argv[3]), centers, dim, ncp, data);
        unsigned C = ncp[0].size();
        FILE* f = fopen(argv[4], "wb");
        fwrite(centers, 4, (size_t)C * dim, f);
        fclose(f);
        std::vector<unsigned> h;
        for (auto& row : ncp) h.insert(h.end(), row.begin(), row.end());
        write_u32(argv[5], h);
        return 0;
    }
    if (mode == "quant" && argc == 5) {
        // quant data.fvecs alpha out.q   (out.q must not exist)
        float* data = nullptr;
        unsigned num = 0, dim = 0;
        int8_t* q = nullptr;
        float* scales = nullptr;
        int* zps = nullptr;
        smart::production_adapter::load_dataset_return_int8_arr_infile(std::string(argv[2]), std::string(argv[4]),
                                                                       data, num, dim, (float)atof(argv[3]), q,
                                                                       scales, zps);
        return 0;
    }
    fprintf(stderr, "usage: bf data attrs queries ranges k out | bf_omp data attrs queries ranges k threads chunk out | cluster data labels centroids hist | "
                    "quant data alpha out.q\n");
    return 2;
}
