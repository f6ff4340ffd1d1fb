// cli.cpp -- command-line front end with the reference's config format and a `--backend b200`.
//
// Usage mirrors the reference CLI (test.cpp:185-357): [--gpu N] [--backend b200] [config_file],
// config = 4 lines (dataset path, k, cluster count, run count; runs defaults to 1 when missing or
// invalid, test.cpp:314-337). A CSV dataset is read by the library in parallel straight into the
// dim-major layout Fit takes (fdb200_read_csv; helper.cpp:9-63, test.cpp:110-115); a path ending in
// .fbin is the binary form (int32 n, int32 d, row-major float32; fdb200_read_fbin). Extra run-time
// switches replace the reference's compile-time ones: --precision fp32|tf32 (USE_CUBLAS_TF32),
// --density laplacian|gaussian (USE_GAUSSIAN_KERNEL), --engine auto|simt|tcgen05. --save-knn FILE
// writes the kNN graph of the first run (fdb200_knn_graph_save) and fits from it; --load-knn FILE
// skips the kNN and fits from a saved graph of at least k ranks (fdb200_knn_graph_load).
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <sstream>
#include <string>
#include <vector>

#include "b200fastdec.h"

static void usage(const char* prog)
{
    printf("Usage: %s [--gpu N] [--backend b200] [--precision fp32|tf32] [--density laplacian|gaussian]\n"
           "          [--engine auto|simt|tcgen05] [--save-knn FILE | --load-knn FILE] [config_file]\n", prog);
    printf("  config_file    4 lines: dataset (CSV, or .fbin binary), k, cluster count, run count\n"
           "                 (default ./config.txt)\n");
}

int main(int argc, char** argv)
{
    std::string cfg_path = "./config.txt";
    FdB200Opts opts;
    fdb200_opts_init(&opts);
    int gpu = 0;
    std::string save_knn, load_knn;
    for (int i = 1; i < argc; ++i) {
        const std::string a = argv[i];
        auto value = [&](const char* flag) -> std::string {
            if (i + 1 >= argc) {
                printf("Error: %s requires a value\n", flag);
                usage(argv[0]);
                exit(EXIT_FAILURE);
            }
            return argv[++i];
        };
        if (a == "--gpu" || a == "-g") gpu = atoi(value("--gpu").c_str());
        else if (a.rfind("--gpu=", 0) == 0) gpu = atoi(a.c_str() + 6);
        else if (a == "--backend" || a == "-b" || a.rfind("--backend=", 0) == 0) {
            const std::string b = (a.rfind("--backend=", 0) == 0) ? a.substr(10) : value("--backend");
            if (b != "b200") {
                printf("Error: invalid backend '%s'. This build provides 'b200'.\n", b.c_str());
                return EXIT_FAILURE;
            }
        } else if (a == "--precision") {
            const std::string v = value("--precision");
            opts.precision = (v == "tf32") ? FDB200_TF32 : FDB200_FP32;
        } else if (a == "--density") {
            const std::string v = value("--density");
            opts.density_kernel = (v == "gaussian") ? FDB200_GAUSSIAN : FDB200_LAPLACIAN;
        } else if (a == "--engine") {
            const std::string v = value("--engine");
            opts.engine = (v == "simt") ? FDB200_ENGINE_SIMT : (v == "tcgen05") ? FDB200_ENGINE_TCGEN05
                                                                              : FDB200_ENGINE_AUTO;
        } else if (a == "--save-knn") {
            save_knn = value("--save-knn");
        } else if (a == "--load-knn") {
            load_knn = value("--load-knn");
        } else if (a == "--help" || a == "-h") {
            usage(argv[0]);
            return EXIT_SUCCESS;
        } else {
            cfg_path = a;
        }
    }

    std::ifstream cf(cfg_path);
    if (!cf) {
        printf("Can't open the file: %s\n", cfg_path.c_str());
        return EXIT_FAILURE;
    }
    std::vector<std::string> lines;
    for (std::string l; std::getline(cf, l);) lines.push_back(l);
    if (lines.size() < 3) {
        printf("Error: the config needs at least 3 lines\n");
        return EXIT_FAILURE;
    }
    const std::string data_file = lines[0];
    const int k = atoi(lines[1].c_str());
    const int c = atoi(lines[2].c_str());
    int runs = 1;
    if (lines.size() >= 4) {
        runs = atoi(lines[3].c_str());
        if (runs < 1) runs = 1;
    }
    printf("Read dataset from: %s\nNumber of nearest neighbors: %d\nNumber of clusters: %d\n"
           "Number of runs: %d\nBackend: b200\n", data_file.c_str(), k, c, runs);

    int n = 0, d = 0;
    const auto tr0 = std::chrono::steady_clock::now();
    const bool fbin = data_file.size() > 5 && data_file.compare(data_file.size() - 5, 5, ".fbin") == 0;
    if ((fbin ? fdb200_fbin_shape(data_file.c_str(), &n, &d) : fdb200_csv_shape(data_file.c_str(), &n, &d)) !=
        FDB200_OK) {
        printf("Error: could not read %s: %s\n", data_file.c_str(), fdb200_last_error());
        return EXIT_FAILURE;
    }
    std::vector<float> dm((size_t)n * d);   // dim-major, as Fit takes it (test.cpp:110-115)
    if ((fbin ? fdb200_read_fbin(data_file.c_str(), n, d, dm.data(), 0)
              : fdb200_read_csv(data_file.c_str(), n, d, dm.data(), 0)) != FDB200_OK) {
        printf("Error: could not read %s: %s\n", data_file.c_str(), fdb200_last_error());
        return EXIT_FAILURE;
    }
    printf("Read %d points of dimension %d in %.3f s\n", n, d,
           std::chrono::duration<double>(std::chrono::steady_clock::now() - tr0).count());
    if (n < k) {
        printf("Error: k value is larger that the number of reference points\n");
        return EXIT_FAILURE;
    }

    // a kNN graph to fit from: loaded (--load-knn), or computed once and saved (--save-knn)
    std::vector<float> gdist;
    std::vector<int> gidx;
    if (!load_knn.empty()) {
        int gn = 0, gk = 0, gflags = 0;
        if (fdb200_knn_graph_shape(load_knn.c_str(), &gn, &gk, &gflags) != FDB200_OK) {
            printf("Error: %s\n", fdb200_last_error());
            return EXIT_FAILURE;
        }
        if (gn != n || gk < k) {
            printf("Error: %s holds %d points x %d ranks; the dataset has %d points and k is %d\n", load_knn.c_str(),
                   gn, gk, n, k);
            return EXIT_FAILURE;
        }
        gdist.resize((size_t)gn * gk);
        gidx.resize((size_t)gn * gk);
        if (fdb200_knn_graph_load(load_knn.c_str(), gn, gk, gdist.data(), gidx.data()) != FDB200_OK) {
            printf("Error: %s\n", fdb200_last_error());
            return EXIT_FAILURE;
        }
        printf("Loaded a kNN graph of %d ranks from %s\n", gk, load_knn.c_str());
    } else if (!save_knn.empty()) {
        gdist.resize((size_t)n * k);
        gidx.resize((size_t)n * k);
        FdB200Opts o = opts;
        o.device = gpu;
        if (fdb200_knn(dm.data(), n, d, k, &o, gdist.data(), gidx.data(), nullptr) != FDB200_OK ||
            fdb200_knn_graph_save(save_knn.c_str(), gdist.data(), gidx.data(), n, k, opts.precision) != FDB200_OK) {
            printf("Error: %s\n", fdb200_last_error());
            return EXIT_FAILURE;
        }
        printf("Saved the kNN graph (%d ranks) to %s\n", k, save_knn.c_str());
    }

    for (int run = 1; run <= runs; ++run) {
        try {
            B200FastDEC model(k, c, "b200_fastdec", gpu, &opts);
            const auto t0 = std::chrono::steady_clock::now();
            if (gdist.empty()) model.Fit(dm.data(), n, d);
            else model.FitFromKnn(dm.data(), n, d, gdist.data(), gidx.data());
            const double wall =
                std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
            const FdB200Stats& st = model.get_stats();
            printf("Finished run %d of B200FastDEC: %.6f s (device: total %.3f ms, kNN %.3f ms, "
                   "density+detection %.3f ms, DC reduction %.3f ms, labels %.3f ms; cores %d, k %d)\n",
                   run, wall, st.total_ms, st.knn_ms, st.density_ms, st.dc_ms, st.labels_ms, st.num_cores,
                   st.final_k);
            printf("Cluster centers found: \nlength: %d\n[", (int)model.get_center_indices().size());
            for (size_t i = 0; i < model.get_center_indices().size(); ++i)
                printf("%s%d", i ? "," : "", model.get_center_indices()[i]);
            printf("]\n\n");
        } catch (const std::exception& e) {
            fprintf(stderr, "%s\n", e.what());
            return EXIT_FAILURE;
        }
    }
    return EXIT_SUCCESS;
}
