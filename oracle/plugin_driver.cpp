// plugin_driver.cpp -- TEST INFRASTRUCTURE. Drives the reference's unmodified FastDECBase::Fit
// (fastdecbase.cpp:159-228, compiled from the reference tree by oracle/Makefile) with the B200 kNN
// plug-in of symwarp-fastdec_b200/integration/b200knnfastdec.h, the way the reference's CLI drives a
// backend (test.cpp:124-140). Depending on the build, DC reduction is the reference's own
// dcreductioncuda.cu or the engine's (integration/b200_dc_reduction.cpp).
//
//   plugin_fit <data.f32: dim-major float32 D x N> N D k c gpu <out.bin>
// out.bin: c int32 centers, then N int32 labels. Exit 0 on success, 2 when Fit throws.
#include <cstdio>
#include <cstdlib>
#include <exception>
#include <vector>

#include "b200knnfastdec.h"

int main(int argc, char** argv)
{
    if (argc != 8) {
        fprintf(stderr, "usage: %s data.f32 N D k c gpu out.bin\n", argv[0]);
        return 1;
    }
    const int n = atoi(argv[2]), d = atoi(argv[3]), k = atoi(argv[4]), c = atoi(argv[5]), gpu = atoi(argv[6]);
    std::vector<float> x((size_t)n * d);
    FILE* f = fopen(argv[1], "rb");
    if (!f || fread(x.data(), sizeof(float), x.size(), f) != x.size()) {
        fprintf(stderr, "could not read %s\n", argv[1]);
        return 1;
    }
    fclose(f);
    try {
        B200KnnFastDEC model(k, c, "b200_knn_plugin", gpu);
        model.Fit(x.data(), n, d);
        const integer_1d_array& ctr = model.get_center_indices();
        const integer_1d_array& lab = model.get_labels();
        std::vector<int> out;
        for (int i = 0; i < c; ++i) out.push_back(i < ctr.length() ? (int)ctr[i] : -1);
        for (int i = 0; i < lab.length(); ++i) out.push_back((int)lab[i]);
        FILE* o = fopen(argv[7], "wb");
        if (!o || fwrite(out.data(), sizeof(int), out.size(), o) != out.size()) return 1;
        fclose(o);
    } catch (const std::exception& e) {
        fprintf(stderr, "%s\n", e.what());
        return 2;
    }
    return 0;
}
