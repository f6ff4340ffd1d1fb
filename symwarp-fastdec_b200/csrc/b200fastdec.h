// b200fastdec.h -- C++ host class with the duck-typed surface the reference's CLI drives
// (test.cpp:124-140): ctor (k, c, name, gpu), Fit(dim-major data, N, D), get_center_indices(),
// get_labels(). It mirrors SymWarpFullGpuFastDEC (full_gpu/symwarpfullgpufastdec.h:8-48) and runs
// the whole fit through the C ABI in include/fastdec_b200.h.
#pragma once

#include <stdexcept>
#include <string>
#include <vector>

#include "fastdec_b200.h"

class B200FastDEC
{
public:
    // Prints the same "- <name> : " banner as FastDECBase::FastDECBase (fastdecbase.cpp:147-153).
    B200FastDEC(int num_k_points, int num_clusters, const char* name, int cuda_device_id = 0,
                const FdB200Opts* opts = nullptr);

    // Throws std::runtime_error with the engine's message on failure; "Fit: not enough core
    // points" is reported exactly as the reference throws it (fastdecbase.cpp:188-191).
    void Fit(const float* data, int num_points, int num_dim);

    // The same fit from a finished kNN graph (host, rank-major, rank stride num_points; its first
    // k ranks are used), e.g. one loaded with fdb200_knn_graph_load: the stages after
    // build_knn_graph (fastdecbase.cpp:173-227) without recomputing the kNN.
    void FitFromKnn(const float* data, int num_points, int num_dim, const float* knn_dist, const int* knn_idx);

    const std::vector<int>& get_center_indices() const { return m_centers; }
    const std::vector<int>& get_labels() const { return m_labels; }
    const std::vector<float>& get_densities() const { return m_densities; }
    const FdB200Stats& get_stats() const { return m_stats; }

private:
    int m_num_k_points;
    int m_num_clusters;
    FdB200Opts m_opts;
    std::vector<int> m_centers;
    std::vector<int> m_labels;
    std::vector<float> m_densities;
    FdB200Stats m_stats;
};
