// b200_dc_reduction.cpp -- reference-side replacement of the DC-reduction entry point. Linked in place of
// the reference's dcreductioncuda.cu, it defines warp_parallel_dc_reduction_cuda with the declaration of
// dcreductioncuda.h:45-51, so FastDECBase::dc_reduction (fastdecbase.cpp:335-356) runs the B200
// engine's DC reduction and center selection (fdb200_dc_reduction) without a change to the reference.
//
// Contract kept: host densities of every point, host core indices, core_nb cores, num_centers
// centers; core_cdh_index_host[i] = nearest strictly denser point of core i (-1 if none) and
// center_indices_host = num_centers global indices (-1 padded); false on bad arguments or failure
// (dcreductioncuda.cu:632-644), which makes FastDECBase throw. The dataset is the Dataset's host copy.
#include <cstdio>

#include "dataset.h"
#include "dcreductioncuda.h"
#include "fastdec_b200.h"

bool warp_parallel_dc_reduction_cuda(Dataset& ds, const float* ds_den_host, const int* core_indices_host,
                                     int core_nb, int num_centers, int* core_cdh_index_host,
                                     int* center_indices_host)
{
    if (core_nb <= 0 || num_centers <= 0 || ds.host_data() == nullptr || ds_den_host == nullptr ||
        core_indices_host == nullptr || core_cdh_index_host == nullptr || center_indices_host == nullptr ||
        ds.dim() <= 0 || ds.num_points() <= 0)
        return false;
    FdB200Opts o;
    fdb200_opts_init(&o);
    o.device = ds.cuda_device_id();
    const int rc = fdb200_dc_reduction(ds.host_data(), ds.num_points(), ds.dim(), ds_den_host, core_indices_host,
                                       core_nb, num_centers, &o, core_cdh_index_host, center_indices_host);
    if (rc != FDB200_OK) fprintf(stderr, "fdb200_dc_reduction: %s\n", fdb200_last_error());
    return rc == FDB200_OK;
}
