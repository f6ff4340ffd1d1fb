// b200fastdec.cpp -- see b200fastdec.h.
#include "b200fastdec.h"

#include <cstdio>
#include <cstring>

B200FastDEC::B200FastDEC(int num_k_points, int num_clusters, const char* name, int cuda_device_id,
                         const FdB200Opts* opts)
    : m_num_k_points(num_k_points), m_num_clusters(num_clusters)
{
    printf("- %-17s : \n", name);
    if (opts) m_opts = *opts;
    else fdb200_opts_init(&m_opts);
    m_opts.device = cuda_device_id;
    std::memset(&m_stats, 0, sizeof(m_stats));
}

void B200FastDEC::Fit(const float* data, int num_points, int num_dim)
{
    m_centers.assign(m_num_clusters > 0 ? m_num_clusters : 0, -1);
    m_labels.assign(num_points > 0 ? num_points : 0, -1);
    m_densities.assign(num_points > 0 ? num_points : 0, 0.0f);
    const int rc = fdb200_fit(data, num_points, num_dim, m_num_k_points, m_num_clusters, &m_opts,
                              m_centers.data(), m_labels.data(), m_densities.data(), &m_stats);
    if (rc != FDB200_OK) throw std::runtime_error(fdb200_last_error());
}

void B200FastDEC::FitFromKnn(const float* data, int num_points, int num_dim, const float* knn_dist,
                             const int* knn_idx)
{
    m_centers.assign(m_num_clusters > 0 ? m_num_clusters : 0, -1);
    m_labels.assign(num_points > 0 ? num_points : 0, -1);
    m_densities.assign(num_points > 0 ? num_points : 0, 0.0f);
    FdB200Opts o = m_opts;
    o.inputs_on_device = 0;
    o.outputs_on_device = 0;
    const int rc = fdb200_fit_from_knn(data, knn_dist, knn_idx, num_points, num_dim, m_num_k_points, m_num_clusters,
                                       &o, m_centers.data(), m_labels.data(), m_densities.data(), &m_stats);
    if (rc != FDB200_OK) throw std::runtime_error(fdb200_last_error());
}
