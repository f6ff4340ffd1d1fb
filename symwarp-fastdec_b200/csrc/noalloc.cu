// noalloc.cu -- fdb200_density_noalloc: the kNN density and its exact mean with no allocation at all.
//
// Working memory is one fixed array in the library image (g_mean_scratch, 6.1 MiB, enough for
// FDB200_NOALLOC_MAX_POINTS points). Its device address is looked up once per device with
// cudaGetSymbolAddress while that device is current, and cached; nothing else is requested from the
// CUDA allocator, the host heap of the runtime, or any library during a call.
#include "fdb_internal.h"

#include <mutex>

namespace fdb {
namespace {

constexpr size_t kScratchBytes = mean_scratch_bytes(FDB200_NOALLOC_MAX_POINTS);

// every word the mean kernels read is written earlier in the same call: nothing here has to start
// at zero
__device__ __align__(256) unsigned char g_mean_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_addr[kMaxDevices] = {};

// The array's address on `device`, looked up on the first call for that device (device current).
// The same one-time set-up also loads every kernel this entry point launches: CUDA loads kernels
// lazily, at their first launch, and a load obtains device memory for the code.
void* scratch_on(int device)
{
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    if (!g_scratch_addr[device]) {
        void* p = nullptr;
        FDB_CUDA(cudaGetSymbolAddress(&p, g_mean_scratch));
        preload_mean_density_kernels();
        g_scratch_addr[device] = p;
    }
    return g_scratch_addr[device];
}

}  // namespace
}  // namespace fdb

extern "C" int fdb200_density_noalloc(const float* knn_dist_dev, int n, int k, const FdB200Opts* opts,
                                      float* densities_dev, double* mean_dev)
{
    using namespace fdb;
    FdB200Opts o;
    fdb200_opts_init(&o);
    if (opts) {
        if (opts->struct_size != (int)sizeof(FdB200Opts)) {
            set_last_error("FdB200Opts.struct_size mismatch: initialise options with fdb200_opts_init");
            return FDB200_EINVAL;
        }
        o = *opts;
    }
    try {
        FDB_REQUIRE(knn_dist_dev && densities_dev && mean_dev && n > 0 && k > 0,
                    "fdb200_density_noalloc: null pointer or n, k < 1");
        FDB_REQUIRE(n <= FDB200_NOALLOC_MAX_POINTS,
                    "fdb200_density_noalloc: n = " + std::to_string(n) + " exceeds the fixed scratch (at most " +
                        std::to_string(FDB200_NOALLOC_MAX_POINTS) + " points); use fdb200_density");
        FDB_REQUIRE(o.device >= 0 && o.device < kMaxDevices, "fdb200_density_noalloc: bad device ordinal");
        int cur = -1;
        FDB_CUDA(cudaGetDevice(&cur));
        struct Restore {   // the caller's current device is left as it was
            int dev;
            bool on;
            ~Restore()
            {
                if (on) cudaSetDevice(dev);
            }
        } restore{cur, cur != o.device};
        if (cur != o.device) FDB_CUDA(cudaSetDevice(o.device));
        void* scratch = scratch_on(o.device);
        cudaStream_t s = (cudaStream_t)o.stream;
        exact_mean_in(scratch, kScratchBytes, knn_dist_dev, n, k, mean_dev, s);
        density_from_mean(knn_dist_dev, n, k, o.density_kernel == FDB200_GAUSSIAN, mean_dev, densities_dev, s);
        set_last_error("");
        return FDB200_OK;
    } catch (const Error& e) {
        set_last_error(e.what());
        return e.code;
    } catch (const std::exception& e) {
        set_last_error(e.what());
        return FDB200_EINTERNAL;
    }
}
