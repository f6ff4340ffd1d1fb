// b200knnfastdec.h -- reference-side kNN plug-in: a FastDECBase backend whose compute_knn runs on the
// B200 engine. Compiles inside the reference tree (it includes fastdecbase.h and dataset.h from
// cyberbull66/symwarp-fastdec) and links libfastdec_b200.so.
//
// FastDECBase::compute_knn (fastdecbase.h:43-46) takes the bound Dataset and caller-allocated host
// outputs of N*k entries and must return them rank-major ([q*N + i]), Euclidean, ascending by
// (d2, index), self excluded; false makes build_knn_graph throw (fastdecbase.cpp:244-248). The symwarp
// backend forwards to symtri_knn_cuda (symwarpfastdec.cpp:4-10); this one forwards to fdb200_knn,
// which has the same contract, on the Dataset's GPU (Dataset::cuda_device_id, dataset.h:30).
// Everything else of FastDECBase::Fit (density, DC detection, k-halving, DC reduction, labels) stays
// the reference's own code.
#pragma once

#include <cstdio>

#include "dataset.h"
#include "fastdec_b200.h"
#include "fastdecbase.h"

class B200KnnFastDEC : public FastDECBase
{
public:
    using FastDECBase::FastDECBase;

    // options for the engine (precision, engine choice); the device comes from the Dataset
    FdB200Opts& options() { return m_opts; }

protected:
    bool compute_knn(Dataset& ds, int k, float* out_knn_dists, int* out_knn_indices) override
    {
        FdB200Opts o = m_opts;
        o.device = ds.cuda_device_id();
        const int rc = fdb200_knn(ds.host_data(), ds.num_points(), ds.dim(), k, &o, out_knn_dists,
                                  out_knn_indices, nullptr);
        if (rc != FDB200_OK) fprintf(stderr, "fdb200_knn: %s\n", fdb200_last_error());
        return rc == FDB200_OK;
    }

private:
    FdB200Opts m_opts = [] {
        FdB200Opts o;
        fdb200_opts_init(&o);
        return o;
    }();
};
