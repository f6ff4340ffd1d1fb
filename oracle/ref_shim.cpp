// ref_shim.cpp -- TEST INFRASTRUCTURE. Links the reference's own host stages (fastdecbase.cpp and
// helper.cpp, compiled in place from the reference tree by oracle/Makefile) with CPU stand-ins
// for the two GPU entry points those stages call, so the reference's density, DC detection,
// k-halving loop and final clustering run unmodified on the host:
//   * Dataset (dataset.h:8-39): host-only Bind/Release; the device copy is never made.
//   * warp_parallel_dc_reduction_cuda (dcreductioncuda.h:45-51): the oracle's CPU restatement.
//   * compute_knn (fastdecbase.h:43-46): the oracle's exact CPU self-kNN.
// Output goes only to oracle/_ref/. Nothing in the product links this file.
#include "fastdecbase.h"
#include "dcreductioncuda.h"
#include "dataset.h"
#include "appexception.h"
#include "fastdec_oracle.h"

#include <cstdlib>
#include <cstring>
#include <thread>
#include <vector>

static int shim_threads()
{
    const char* t = getenv("FASTDEC_ORACLE_THREADS");
    int n = t ? atoi(t) : 0;
    if (n <= 0) n = (int)std::thread::hardware_concurrency();
    return n > 0 ? n : 1;
}

Dataset::~Dataset() { Release(); }

void Dataset::Bind(const float* host_data, int num_points, int dim, int cuda_device_id)
{
    Release();
    m_host_data = host_data;
    m_num_points = num_points;
    m_dim = dim;
    m_cuda_device_id = cuda_device_id;
}

bool Dataset::EnsureUploaded() { return false; }

void Dataset::Release()
{
    m_device_data = nullptr;
    m_device_pitch_bytes = 0;
}

bool warp_parallel_dc_reduction_cuda(Dataset& ds, const float* ds_den_host, const int* core_indices_host,
                                     int core_nb, int num_centers, int* core_cdh_index_host,
                                     int* center_indices_host)
{
    if (core_nb <= 0 || num_centers <= 0 || ds.host_data() == nullptr || ds_den_host == nullptr ||
        core_indices_host == nullptr || core_cdh_index_host == nullptr || center_indices_host == nullptr ||
        ds.dim() <= 0 || ds.num_points() <= 0)
        return false;
    std::vector<float> delta(core_nb);
    std::vector<int> rank(core_nb);
    return or_dc_reduction(ds.host_data(), ds.num_points(), ds.dim(), ds_den_host, core_indices_host,
                           core_nb, num_centers, shim_threads(), core_cdh_index_host, delta.data(),
                           rank.data(), center_indices_host) == 0;
}

namespace {

// compute_knn is the oracle's exact CPU kNN, or -- when given_dist / given_idx are set -- a copy of
// lists the caller already has (rank-major, k ranks, the layout compute_knn returns), so the
// reference's own stages can be run on another engine's kNN graph
class CpuKnnFastDEC : public FastDECBase
{
public:
    CpuKnnFastDEC(int k, int c, const float* given_dist = nullptr, const int* given_idx = nullptr)
        : FastDECBase(k, c, "oracle_ref_cpu"), m_given_dist(given_dist), m_given_idx(given_idx)
    {
    }
    const real_1d_array& densities() const { return m_densities; }
    const integer_1d_array& parents() const { return m_cdh_ids; }
    int final_k() const { return m_num_k_points; }

protected:
    bool compute_knn(Dataset& ds, int k, float* out_dists, int* out_idx) override
    {
        if (m_given_dist && m_given_idx) {
            const size_t count = (size_t)ds.num_points() * k;
            std::memcpy(out_dists, m_given_dist, count * sizeof(float));
            std::memcpy(out_idx, m_given_idx, count * sizeof(int));
            return true;
        }
        return or_knn(ds.host_data(), ds.num_points(), ds.dim(), k, shim_threads(), out_dists, out_idx) == 0;
    }

private:
    const float* m_given_dist;
    const int* m_given_idx;
};

int run_fit(CpuKnnFastDEC& model, const float* x_dm, int n, int d, int c, int* centers, int* labels,
            float* densities, int* parents, int* cores, int* num_cores, int* final_k, char* err, int err_len);

}  // namespace

// Runs the reference FastDECBase::Fit (fastdecbase.cpp:159-228). Any of the output pointers
// may be null. Returns 0 on success, -2 when the reference throws (message in err if given).
extern "C" int ref_fit(const float* x_dm, int n, int d, int k, int c, int* centers, int* labels,
                       float* densities, int* parents, int* cores, int* num_cores, int* final_k,
                       char* err, int err_len)
{
    CpuKnnFastDEC model(k, c);
    return run_fit(model, x_dm, n, d, c, centers, labels, densities, parents, cores, num_cores, final_k, err,
                   err_len);
}

// The same Fit on a kNN graph the caller supplies (rank-major knn_dist / knn_idx, k ranks of n
// points): everything after build_knn_graph is the reference's own code.
extern "C" int ref_fit_from_knn(const float* x_dm, int n, int d, int k, int c, const float* knn_dist,
                                const int* knn_idx, int* centers, int* labels, float* densities, int* parents,
                                int* cores, int* num_cores, int* final_k, char* err, int err_len)
{
    CpuKnnFastDEC model(k, c, knn_dist, knn_idx);
    return run_fit(model, x_dm, n, d, c, centers, labels, densities, parents, cores, num_cores, final_k, err,
                   err_len);
}

namespace {

int run_fit(CpuKnnFastDEC& model, const float* x_dm, int n, int d, int c, int* centers, int* labels,
            float* densities, int* parents, int* cores, int* num_cores, int* final_k, char* err, int err_len)
{
    try {
        model.Fit(x_dm, n, d);
        const integer_1d_array& ctr = model.get_center_indices();
        const integer_1d_array& lab = model.get_labels();
        const integer_1d_array& cor = model.get_core_indices();
        if (centers) for (int i = 0; i < ctr.length() && i < c; ++i) centers[i] = ctr[i];
        if (labels) for (int i = 0; i < lab.length(); ++i) labels[i] = lab[i];
        if (densities) for (int i = 0; i < model.densities().length(); ++i) densities[i] = model.densities()[i];
        if (parents) for (int i = 0; i < model.parents().length(); ++i) parents[i] = model.parents()[i];
        if (cores) for (int i = 0; i < cor.length(); ++i) cores[i] = cor[i];
        if (num_cores) *num_cores = cor.length();
        if (final_k) *final_k = model.final_k();
        return 0;
    } catch (const std::exception& e) {
        if (err && err_len > 0) {
            strncpy(err, e.what(), (size_t)err_len - 1);
            err[err_len - 1] = '\0';
        }
        return -2;
    }
}

}  // namespace
