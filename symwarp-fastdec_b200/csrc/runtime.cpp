// runtime.cpp -- per-device workspace, error plumbing and stage timing for the C ABI.
//
// The reference allocates and frees every buffer inside each call and runs on the legacy default
// stream (symtriknncuda.cu:367-376, 601-613). Here each device keeps a grow-only workspace across
// calls (the 1.29M-point fit needs ~4 GB of lists and candidate buffers; reallocating them per
// call would cost more than the merge kernels) and work runs on one stream per call.
#include "fdb_internal.h"

#include <map>
#include <memory>

namespace fdb {

static thread_local std::string t_last_error;
thread_local long long g_launches = 0;
thread_local int last_call_launches = 0;

void set_last_error(const std::string& msg) { t_last_error = msg; }

void* DevBuf::ensure(size_t need)
{
    if (need == 0) need = 16;
    if (need <= bytes) return ptr;
    release();
    // round up so slightly larger follow-up requests reuse the allocation
    size_t want = need + need / 8;
    want = (want + 255) & ~size_t(255);
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, want);
    if (e != cudaSuccess) {
        cudaGetLastError();
        e = cudaMalloc(&p, need);
        if (e != cudaSuccess) {
            cudaGetLastError();
            throw Error(FDB200_ENOMEM, "cudaMalloc of " + std::to_string(need) + " bytes failed: " +
                                           cudaGetErrorString(e));
        }
        want = need;
    }
    ptr = p;
    bytes = want;
    return ptr;
}

void DevBuf::release()
{
    if (ptr) cudaFree(ptr);
    ptr = nullptr;
    bytes = 0;
}

void Workspace::release_all()
{
    for (DevBuf* b : {&data, &norms, &lists, &thr, &fthr, &cand, &cnt, &flags, &dist, &idx, &den,
                      &parent, &cores, &scan, &mean_tmp, &dc_tmp, &dc_sel, &labels_tmp, &misc, &ops, &misc2, &spill})
        b->release();
}

Workspace& workspace(int device)
{
    static std::mutex registry_mu;
    static std::map<int, std::unique_ptr<Workspace>> registry;
    std::lock_guard<std::mutex> lk(registry_mu);
    auto& slot = registry[device];
    if (!slot) {
        slot.reset(new Workspace());
        slot->device = device;
    }
    return *slot;
}

int guarded(const FdB200Opts* opts, FdB200Opts* resolved, Workspace** ws_out,
            const std::function<void(Workspace&, const FdB200Opts&, cudaStream_t)>& fn)
{
    FdB200Opts o;
    fdb200_opts_init(&o);
    if (opts) {
        if (opts->struct_size != (int)sizeof(FdB200Opts)) {
            set_last_error("FdB200Opts.struct_size mismatch: initialise options with fdb200_opts_init");
            return FDB200_EINVAL;
        }
        o = *opts;
    }
    if (resolved) *resolved = o;
    try {
        int count = 0;
        FDB_CUDA(cudaGetDeviceCount(&count));
        // Dataset::EnsureUploaded / select_cuda_device reject a bad index (knndcshared.h:39-57)
        FDB_REQUIRE(o.device >= 0 && o.device < count,
                    "device " + std::to_string(o.device) + " out of range (" + std::to_string(count) +
                        " CUDA device(s))");
        FDB_CUDA(cudaSetDevice(o.device));
        Workspace& ws = workspace(o.device);
        std::lock_guard<std::mutex> lk(ws.mu);
        if (!ws.own_stream) FDB_CUDA(cudaStreamCreateWithFlags(&ws.own_stream, cudaStreamNonBlocking));
        if (!ws.pinned) FDB_CUDA(cudaMallocHost((void**)&ws.pinned, 64 * sizeof(int)));
        cudaStream_t s = o.stream ? (cudaStream_t)o.stream : ws.own_stream;
        if (ws_out) *ws_out = &ws;
        const long long launches0 = g_launches;
        fn(ws, o, s);
        last_call_launches = (int)(g_launches - launches0);
        set_last_error("");
        return FDB200_OK;
    } catch (const Error& e) {
        set_last_error(e.what());
        return e.code;
    } catch (const std::bad_alloc&) {
        set_last_error("host allocation failed");
        return FDB200_ENOMEM;
    } catch (const std::exception& e) {
        set_last_error(e.what());
        return FDB200_EINTERNAL;
    }
}

StageTimer::StageTimer(cudaStream_t st) : s(st)
{
    for (auto& e : ev) e = nullptr;
}

StageTimer::~StageTimer()
{
    for (int i = 0; i < n; ++i)
        if (ev[i]) cudaEventDestroy(ev[i]);
}

int StageTimer::mark()
{
    if (n >= 32) throw Error(FDB200_EINTERNAL, "stage timer overflow");
    FDB_CUDA(cudaEventCreate(&ev[n]));
    FDB_CUDA(cudaEventRecord(ev[n], s));
    return n++;
}

double StageTimer::ms(int a, int b)
{
    FDB_CUDA(cudaEventSynchronize(ev[b]));
    float t = 0.0f;
    FDB_CUDA(cudaEventElapsedTime(&t, ev[a], ev[b]));
    return (double)t;
}

}  // namespace fdb

extern "C" const char* fdb200_last_error(void) { return fdb::t_last_error.c_str(); }
