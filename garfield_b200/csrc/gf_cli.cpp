// realdataset_search / normaldataset_search: the reference's experiment CLI over the
// garfield_b200 C ABI.  Same flags as realdataset_search.cu:2712-2751 (README.md:101-170),
// same result CSV columns (realdataset_search.cu:2440,2509):
//   ef,recall,qps,total_cost,cost1,cost2,cost3,kernal_cost
// cost1 = cell intersection + ordering (one planning call), cost2 = 0 (folded into
// cost1), cost3 = search kernel; all in seconds, measured with CUDA events.
// qps = qnum / (cost1 + cost2 + cost3) as in realdataset_search.cu:2506-2508.
// Extra flags: --ef "10,20,..." (default: the reference's 33-value sweep), --k,
// --width, --device, --max_iter, --exact_tc (exact route on the tensor cores), --route 1
// (route each query by cost: graph walk or tensor-core exact scan).
// Invoked as normaldataset_search (normaldataset_search.cu:1748-2104) the grid is
// uniform instead of read from --grid: --shape "16" (slices per attribute, the
// reference's compiled-in default) over [--domain_lo, --domain_hi) = [0, 1e6), and the
// graph degree defaults to 16 (the reference fixes it there).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <strings.h>
#include <vector>

#include "garfield.h"

namespace {

int die(const char* what, gf_status s) {
    fprintf(stderr, "%s: %s (%s)\n", what, gf_status_string(s), gf_last_error());
    return 1;
}

std::vector<uint32_t> parse_list(const std::string& s) {
    std::vector<uint32_t> v;
    size_t i = 0;
    while (i < s.size()) {
        size_t j = s.find(',', i);
        if (j == std::string::npos) j = s.size();
        if (j > i) v.push_back((uint32_t)std::stoul(s.substr(i, j - i)));
        i = j + 1;
    }
    return v;
}

}  // namespace

int main(int argc, char** argv) {
    std::string data, query, range, gt, cprefix, csuffix = ".cagra32", global, grid, attrs, cluster, result = "result.csv";
    float prefilter = 0.0f, f2h = 1.0f;
    uint32_t postfilter = 0xFFFFFFFFu, degree = 32, k = 10, width = 1, max_iter = 10000, exact_tc = 0, route = 0;
    int device = 0;
    std::string prog = argv[0];
    const bool normal = prog.size() >= 20 && prog.compare(prog.size() - 20, 20, "normaldataset_search") == 0;
    std::vector<uint32_t> shape = {16};
    float domain_lo = 0.0f, domain_hi = 1000000.0f;
    if (normal) degree = 16;
    // realdataset_search.cu:2757-2760, ascending
    std::vector<uint32_t> ef = {10,  10,  15,  20,  25,  30,  35,  40,  45,  50,   55,   60,   70,   80,   90,   100, 120,
                                140, 160, 180, 200, 250, 300, 400, 500, 600, 700, 800, 900, 1000, 1100, 1400, 1700};
    for (int i = 1; i + 1 < argc; ++i) {
        std::string a = argv[i], v = argv[i + 1];
        if (a == "--data_path") data = v;
        else if (a == "--query_path") query = v;
        else if (a == "--range") range = v;
        else if (a == "--gt") gt = v;
        else if (a == "--cagra_prefix") cprefix = v;
        else if (a == "--cagra_suffix") csuffix = v;
        else if (a == "--global_graph") global = v;
        else if (a == "--grid") grid = v;
        else if (a == "--attrs") attrs = v;
        else if (a == "--cluster") cluster = v;
        else if (a == "--result") result = v;
        else if (a == "--prefilter") prefilter = std::stof(v);
        else if (a == "--postfilter") postfilter = (uint32_t)std::stoul(v);
        else if (a == "--f2h_factor") f2h = std::stof(v);
        else if (a == "--degree") degree = (uint32_t)std::stoul(v);
        else if (a == "--ef") ef = parse_list(v);
        else if (a == "--k") k = (uint32_t)std::stoul(v);
        else if (a == "--width") width = (uint32_t)std::stoul(v);
        else if (a == "--max_iter") max_iter = (uint32_t)std::stoul(v);
        else if (a == "--exact_tc") exact_tc = (uint32_t)std::stoul(v);
        else if (a == "--route") route = (uint32_t)std::stoul(v);
        else if (a == "--device") device = std::stoi(v);
        else if (a == "--shape") shape = parse_list(v);
        else if (a == "--domain_lo") domain_lo = std::stof(v);
        else if (a == "--domain_hi") domain_hi = std::stof(v);
        else continue;
        ++i;
    }
    if (data.empty() || query.empty() || range.empty() || gt.empty() || cprefix.empty() || global.empty() ||
        (grid.empty() && !normal) || attrs.empty()) {
        fprintf(stderr,
                "usage: %s --data_path F --query_path F --range F --gt F --cagra_prefix P --cagra_suffix S "
                "--global_graph F --grid F --attrs F [--cluster F] [--result F] [--prefilter x] [--postfilter n] "
                "[--f2h_factor a] [--degree R] [--ef l1,l2,..] [--k K] [--width W] [--device d] [--exact_tc 0|1] "
                "[--route 0|1]\n",
                argv[0]);
        return 2;
    }
    gf_index_files fs;
    memset(&fs, 0, sizeof(fs));
    fs.data_path = data.c_str();
    if (route) exact_tc = 1;            // routing by cost sends queries to the tensor-core exact scan
    fs.keep_fp32 = exact_tc ? 1u : 0u;  // the tensor-core exact route reads the fp32 rows
    fs.cagra_prefix = cprefix.c_str();
    fs.cagra_suffix = csuffix.c_str();
    fs.global_graph = global.c_str();
    fs.grid = normal ? nullptr : grid.c_str();  // normaldataset_search ignores --grid
    fs.uniform_dims = (uint32_t)shape.size();
    fs.uniform_shape = shape.data();
    fs.uniform_lo = domain_lo;
    fs.uniform_hi = domain_hi;
    fs.attrs = attrs.c_str();
    fs.cluster = cluster.empty() ? nullptr : cluster.c_str();
    fs.degree = degree;
    fs.f2h_factor = f2h;
    gf_index* idx = nullptr;
    gf_status st = gf_index_open(&fs, device, &idx);
    if (st != GF_OK) return die("gf_index_open", st);
    gf_index_info info;
    gf_index_info_get(idx, &info);
    float* qv = nullptr;
    uint32_t qnum = 0, qdim = 0;
    if ((st = gf_read_fvecs(query.c_str(), &qv, &qnum, &qdim)) != GF_OK) return die("queries", st);
    if (qdim != info.dim) {
        fprintf(stderr, "query dimension %u differs from data dimension %u\n", qdim, info.dim);
        return 1;
    }
    const uint32_t a = info.n_attr;
    std::vector<int32_t> li((size_t)qnum * a), ri((size_t)qnum * a);
    if ((st = gf_read_ranges(range.c_str(), qnum, a, li.data(), ri.data())) != GF_OK) return die("ranges", st);
    std::vector<float> lf(li.begin(), li.end()), rf(ri.begin(), ri.end());
    uint32_t *gtv = nullptr, gq = 0, gk = 0;
    if ((st = gf_read_u32mat(gt.c_str(), &gtv, &gq, &gk)) != GF_OK) return die("ground truth", st);
    if (gq < qnum) {
        fprintf(stderr, "ground truth has %u rows for %u queries\n", gq, qnum);
        return 1;
    }
    cudaSetDevice(device);
    float *dq, *dl, *dr;
    uint32_t* dids;
    cudaMalloc(&dq, sizeof(float) * qnum * qdim);
    cudaMalloc(&dl, sizeof(float) * qnum * a);
    cudaMalloc(&dr, sizeof(float) * qnum * a);
    cudaMalloc(&dids, sizeof(uint32_t) * qnum * k);
    cudaMemcpy(dq, qv, sizeof(float) * qnum * qdim, cudaMemcpyHostToDevice);
    cudaMemcpy(dl, lf.data(), sizeof(float) * qnum * a, cudaMemcpyHostToDevice);
    cudaMemcpy(dr, rf.data(), sizeof(float) * qnum * a, cudaMemcpyHostToDevice);
    gf_plan* plan = nullptr;
    if ((st = gf_plan_create(idx, qnum, &plan)) != GF_OK) return die("gf_plan_create", st);
    FILE* out = fopen(result.c_str(), "w");
    if (!out) {
        fprintf(stderr, "cannot create %s\n", result.c_str());
        return 1;
    }
    fprintf(out, "ef,recall,qps,total_cost,cost1,cost2,cost3,kernal_cost\n");
    cudaEvent_t e0, e1, e2;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    cudaEventCreate(&e2);
    std::vector<uint32_t> res((size_t)qnum * k);
    for (uint32_t L : ef) {
        if (L < k) continue;
        gf_search_params p;
        gf_search_defaults(&p);
        p.L = L;
        p.k = k;
        p.width = width;
        p.max_iter = max_iter;
        p.postfilter = postfilter;
        p.exact_tc = exact_tc;
        p.route = route;
        cudaEventRecord(e0, 0);
        if ((st = gf_plan_queries(idx, plan, dq, dl, dr, qnum, prefilter, nullptr)) != GF_OK) return die("plan", st);
        cudaEventRecord(e1, 0);
        if ((st = gf_search(idx, plan, &p, dids, nullptr, nullptr)) != GF_OK) return die("search", st);
        cudaEventRecord(e2, 0);
        cudaEventSynchronize(e2);
        float ms_plan = 0, ms_search = 0;
        cudaEventElapsedTime(&ms_plan, e0, e1);
        cudaEventElapsedTime(&ms_search, e1, e2);
        cudaMemcpy(res.data(), dids, sizeof(uint32_t) * qnum * k, cudaMemcpyDeviceToHost);
        double recall = 0;
        for (uint32_t q = 0; q < qnum; ++q) {
            uint32_t ng = 0, hit = 0;
            for (uint32_t j = 0; j < gk; ++j) {
                uint32_t g = gtv[(size_t)q * gk + j];
                if (g == GF_NO_ID) continue;
                ++ng;
                for (uint32_t i = 0; i < k; ++i)
                    if (res[(size_t)q * k + i] == g) {
                        ++hit;
                        break;
                    }
            }
            recall += ng ? (double)hit / ng : 1.0;
        }
        recall /= qnum;
        double c1 = ms_plan / 1e3, c3 = ms_search / 1e3, total = c1 + c3;
        fprintf(out, "%u,%.6f,%.3f,%.6f,%.6f,%.6f,%.6f,%.6f\n", L, recall, qnum / total, total, c1, 0.0, c3, c3);
        printf("L=%u recall=%.4f qps=%.1f plan=%.3fms search=%.3fms\n", L, recall, qnum / total, ms_plan, ms_search);
        fflush(stdout);
    }
    fclose(out);
    gf_plan_destroy(plan);
    gf_index_destroy(idx);
    gf_free(qv);
    gf_free(gtv);
    return 0;
}
