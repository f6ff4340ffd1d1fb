// capi.cpp -- the extern "C" boundary (include/fastdec_b200.h) and the Fit orchestration.
//
// Stage order follows FastDECBase::Fit (fastdecbase.cpp:159-228) and SymWarpFullGpuFastDEC::Fit
// (full_gpu/symwarpfullgpufastdec.cpp:31-104): kNN -> density -> DC detection -> k-halving retry
// while cores < c -> centers = cores when equal, else DC reduction -> labels. Unlike the
// reference's fullgpu path there is no host round trip of the kNN lists, densities or core
// indices between stages; the only device->host traffic inside a fit is the core count per
// detection pass, one flag per kNN round and the outputs.
#include "fdb_internal.h"

#include <cstring>

using namespace fdb;

namespace {

const float* upload_f32(DevBuf& buf, const float* src, size_t count, const FdB200Opts& o, cudaStream_t s)
{
    if (o.inputs_on_device) return src;
    float* dst = buf.as<float>(count);
    FDB_CUDA(cudaMemcpyAsync(dst, src, sizeof(float) * count, cudaMemcpyHostToDevice, s));
    return dst;
}

const int* upload_i32(DevBuf& buf, const int* src, size_t count, const FdB200Opts& o, cudaStream_t s)
{
    if (o.inputs_on_device) return src;
    int* dst = buf.as<int>(count);
    FDB_CUDA(cudaMemcpyAsync(dst, src, sizeof(int) * count, cudaMemcpyHostToDevice, s));
    return dst;
}

void download(void* dst, const void* src, size_t bytes, const FdB200Opts& o, cudaStream_t s)
{
    if (!dst || bytes == 0) return;
    FDB_CUDA(cudaMemcpyAsync(dst, src, bytes, o.outputs_on_device ? cudaMemcpyDeviceToDevice
                                                                   : cudaMemcpyDeviceToHost, s));
}

KnnConfig knn_config(int n, int d, int k, const FdB200Opts& o)
{
    KnnConfig c;
    c.n = n;
    c.d = d;
    c.k = k;
    c.ldx = n;
    c.precision = o.precision;
    c.engine = o.engine;
    c.shard_rank = o.shard_rank;
    c.shard_count = o.shard_count;
    c.cand_capacity = o.cand_capacity;
    c.block_lo = o.shard_block_lo;
    c.block_hi = o.shard_block_hi;
    return c;
}

// the configuration of fdb200_knn_partial: as above, plus the symmetric shards' round hook (the other
// entry points run the whole triangle on one device and ignore it)
KnnConfig knn_partial_config(int n, int d, int k, const FdB200Opts& o)
{
    KnnConfig c = knn_config(n, d, k, o);
    c.round_hook = o.round_hook;
    c.round_hook_ctx = o.round_hook_ctx;
    return c;
}

struct FitBuffers {
    double* mean;
    int* centers;
    int* labels;
    int* core_parent;
};

FitBuffers carve(Workspace& ws, int n, int c)
{
    char* base = (char*)ws.misc.ensure(64 + sizeof(int) * (2 * (size_t)n + (size_t)c + 64));
    FitBuffers b;
    b.mean = (double*)base;
    b.centers = (int*)(base + 64);
    b.labels = b.centers + c + 16;
    b.core_parent = b.labels + n + 16;
    return b;
}

// everything after build_knn_graph (fastdecbase.cpp:173-227); dist / idx rank-major on the device
void fit_after_knn(Workspace& ws, const float* x, int n, int d, const float* dist, const int* idx, int k,
                   int c, bool norms_ready, const FdB200Opts& o, cudaStream_t s, int* centers_out,
                   int* labels_out, float* den_out, FdB200Stats* st, StageTimer& tm)
{
    FitBuffers b = carve(ws, n, c);
    float* den = ws.den.as<float>(n);
    int* parent = ws.parent.as<int>(n);
    int* cores = ws.cores.as<int>(n);
    const int gauss = (o.density_kernel == FDB200_GAUSSIAN) ? 1 : 0;

    const int e0 = tm.mark();
    int kk = k;
    exact_mean(ws, dist, n, kk, b.mean, s);
    density_from_mean(dist, n, kk, gauss, b.mean, den, s);
    int nc = dc_detection(ws, idx, den, n, kk, parent, cores, s);
    while (nc < c) {
        if (kk <= 1) throw Error(FDB200_ECORES, "Fit: not enough core points");
        kk /= 2;   // the lists keep their first kk ranks (fastdecbase.cpp:193-198)
        exact_mean(ws, dist, n, kk, b.mean, s);
        density_from_mean(dist, n, kk, gauss, b.mean, den, s);
        nc = dc_detection(ws, idx, den, n, kk, parent, cores, s);
    }
    const int e1 = tm.mark();
    if (nc == c) {
        FDB_CUDA(cudaMemcpyAsync(b.centers, cores, sizeof(int) * c, cudaMemcpyDeviceToDevice, s));
    } else {
        float* norms = ws.norms.as<float>(n);
        if (!norms_ready) compute_norms(x, n, n, d, norms, s);
        dc_reduction(ws, x, n, n, d, norms, den, cores, nc, c, b.core_parent, b.centers, s);
        scatter_core_parents(cores, b.core_parent, nc, parent, s);
    }
    const int e2 = tm.mark();
    final_cluster(ws, parent, n, b.centers, c, b.labels, s);
    download(centers_out, b.centers, sizeof(int) * c, o, s);
    download(labels_out, b.labels, sizeof(int) * n, o, s);
    download(den_out, den, sizeof(float) * n, o, s);
    const int e3 = tm.mark();
    FDB_CUDA(cudaStreamSynchronize(s));
    if (st) {
        st->density_ms = tm.ms(e0, e1);
        st->dc_ms = tm.ms(e1, e2);
        st->labels_ms = tm.ms(e2, e3);
        st->num_cores = nc;
        st->final_k = kk;
    }
}

void fill_knn_stats(FdB200Stats* st, const KnnResult& r)
{
    if (!st) return;
    st->knn_tile_ms = r.tile_ms;
    st->pairs = r.pairs;
    st->candidates = r.candidates;
    st->rounds = r.rounds;
    st->overflow_reruns = r.overflow_reruns;
    st->engine_used = r.engine_used;
}

}  // namespace

extern "C" {

int fdb200_abi_version(void) { return FDB200_ABI_VERSION; }

int fdb200_opts_init(FdB200Opts* opts)
{
    if (!opts) return FDB200_EINVAL;
    std::memset(opts, 0, sizeof(*opts));
    opts->struct_size = (int)sizeof(FdB200Opts);
    opts->device = 0;
    opts->precision = FDB200_FP32;
    opts->density_kernel = FDB200_LAPLACIAN;
    opts->engine = FDB200_ENGINE_AUTO;
    opts->shard_rank = 0;
    opts->shard_count = 1;
    opts->shard_block_lo = -1;
    opts->shard_block_hi = -1;
    return FDB200_OK;
}

int fdb200_knn(const float* data, int n, int d, int k, const FdB200Opts* opts, float* out_dist,
               int* out_idx, FdB200Stats* stats)
{
    if (stats) std::memset(stats, 0, sizeof(*stats));
    if (n <= 1 || k <= 0) return FDB200_OK;   // symtriknncuda.cu:319-321
    const int rc = guarded(opts, nullptr, nullptr, [&](Workspace& ws, const FdB200Opts& o, cudaStream_t s) {
        FDB_REQUIRE(data && out_dist && out_idx, "fdb200_knn: null pointer");
        FDB_REQUIRE(d >= 1, "fdb200_knn: d must be >= 1");
        FDB_REQUIRE(k < n, "fdb200_knn: k must be smaller than n (symtriknncuda.cu:322-324)");
        StageTimer tm(s);
        const int a = tm.mark();
        const float* x = upload_f32(ws.data, data, (size_t)n * d, o, s);
        const int b = tm.mark();
        KnnResult r = knn_lists(ws, x, knn_config(n, d, k, o), s);
        float* dist = o.outputs_on_device ? out_dist : ws.dist.as<float>((size_t)n * k);
        int* idx = o.outputs_on_device ? out_idx : ws.idx.as<int>((size_t)n * k);
        lists_to_rank_major(r.lists, n, k, dist, idx, s);
        const int c = tm.mark();
        if (!o.outputs_on_device) {
            download(out_dist, dist, sizeof(float) * (size_t)n * k, o, s);
            download(out_idx, idx, sizeof(int) * (size_t)n * k, o, s);
        }
        const int e = tm.mark();
        FDB_CUDA(cudaStreamSynchronize(s));
        if (stats) {
            fill_knn_stats(stats, r);
            stats->upload_ms = tm.ms(a, b);
            stats->knn_ms = tm.ms(b, c);
            stats->total_ms = tm.ms(a, e);
        }
    });
    if (stats) stats->launches = last_call_launches;
    return rc;
}

int fdb200_fit(const float* data, int n, int d, int k, int c, const FdB200Opts* opts, int* centers_out,
               int* labels_out, float* densities_out, FdB200Stats* stats)
{
    if (stats) std::memset(stats, 0, sizeof(*stats));
    const int rc = guarded(opts, nullptr, nullptr, [&](Workspace& ws, const FdB200Opts& o, cudaStream_t s) {
        FDB_REQUIRE(data && centers_out && labels_out, "fdb200_fit: null pointer");
        FDB_REQUIRE(n >= 2 && d >= 1 && c >= 1 && k >= 1, "fdb200_fit: need n >= 2, d >= 1, k >= 1, c >= 1");
        FDB_REQUIRE(k < n, "fdb200_fit: k must be smaller than n (symtriknncuda.cu:322-324)");
        StageTimer tm(s);
        const int a = tm.mark();
        const float* x = upload_f32(ws.data, data, (size_t)n * d, o, s);
        const int b = tm.mark();
        KnnResult r = knn_lists(ws, x, knn_config(n, d, k, o), s);
        float* dist = ws.dist.as<float>((size_t)n * k);
        int* idx = ws.idx.as<int>((size_t)n * k);
        lists_to_rank_major(r.lists, n, k, dist, idx, s);
        const int e = tm.mark();
        fit_after_knn(ws, x, n, d, dist, idx, k, c, true, o, s, centers_out, labels_out, densities_out,
                      stats, tm);
        const int f = tm.mark();
        FDB_CUDA(cudaStreamSynchronize(s));
        if (stats) {
            fill_knn_stats(stats, r);
            stats->upload_ms = tm.ms(a, b);
            stats->knn_ms = tm.ms(b, e);
            stats->total_ms = tm.ms(a, f);
        }
    });
    if (stats) stats->launches = last_call_launches;
    return rc;
}

int fdb200_fit_from_knn(const float* data, const float* knn_dist, const int* knn_idx, int n, int d, int k, int c,
                        const FdB200Opts* opts, int* centers_out, int* labels_out, float* densities_out,
                        FdB200Stats* stats)
{
    if (stats) std::memset(stats, 0, sizeof(*stats));
    const int rc = guarded(opts, nullptr, nullptr, [&](Workspace& ws, const FdB200Opts& o, cudaStream_t s) {
        FDB_REQUIRE(data && knn_dist && knn_idx && centers_out && labels_out, "fdb200_fit_from_knn: null pointer");
        FDB_REQUIRE(n >= 2 && d >= 1 && c >= 1 && k >= 1 && k < n, "fdb200_fit_from_knn: bad sizes");
        StageTimer tm(s);
        const int a = tm.mark();
        const float* x = upload_f32(ws.data, data, (size_t)n * d, o, s);
        // the first k ranks of the graph (rank stride n)
        const float* dist = upload_f32(ws.dist, knn_dist, (size_t)n * k, o, s);
        const int* idx = upload_i32(ws.idx, knn_idx, (size_t)n * k, o, s);
        fit_after_knn(ws, x, n, d, dist, idx, k, c, false, o, s, centers_out, labels_out, densities_out, stats, tm);
        const int f = tm.mark();
        FDB_CUDA(cudaStreamSynchronize(s));
        if (stats) stats->total_ms = tm.ms(a, f);
    });
    if (stats) stats->launches = last_call_launches;
    return rc;
}

int fdb200_dc_reduction(const float* data, int n, int d, const float* densities, const int* core_indices,
                        int core_nb, int num_centers, const FdB200Opts* opts, int* core_parent_out,
                        int* centers_out)
{
    return guarded(opts, nullptr, nullptr, [&](Workspace& ws, const FdB200Opts& o, cudaStream_t s) {
        // dcreductioncuda.cu:632-644 argument checks
        FDB_REQUIRE(core_nb > 0 && num_centers > 0 && data && densities && core_indices && core_parent_out &&
                        centers_out && d > 0 && n > 0,
                    "fdb200_dc_reduction: bad arguments");
        const float* x = upload_f32(ws.data, data, (size_t)n * d, o, s);
        const float* den = upload_f32(ws.den, densities, (size_t)n, o, s);
        const int* cores = upload_i32(ws.cores, core_indices, (size_t)core_nb, o, s);
        if (!o.inputs_on_device) {
            for (int i = 0; i < core_nb; ++i)
                FDB_REQUIRE(core_indices[i] >= 0 && core_indices[i] < n, "fdb200_dc_reduction: core index out of range");
        }
        float* norms = ws.norms.as<float>(n);
        compute_norms(x, n, n, d, norms, s);
        FitBuffers b = carve(ws, core_nb, num_centers);
        dc_reduction(ws, x, n, n, d, norms, den, cores, core_nb, num_centers, b.core_parent, b.centers, s);
        download(core_parent_out, b.core_parent, sizeof(int) * core_nb, o, s);
        download(centers_out, b.centers, sizeof(int) * num_centers, o, s);
        FDB_CUDA(cudaStreamSynchronize(s));
    });
}

int fdb200_density(const float* knn_dist, int n, int k, const FdB200Opts* opts, float* densities_out,
                   double* mean_out)
{
    return guarded(opts, nullptr, nullptr, [&](Workspace& ws, const FdB200Opts& o, cudaStream_t s) {
        FDB_REQUIRE(knn_dist && densities_out && n > 0 && k > 0, "fdb200_density: bad arguments");
        const float* dist = upload_f32(ws.dist, knn_dist, (size_t)n * k, o, s);
        FitBuffers b = carve(ws, n, 1);
        float* den = o.outputs_on_device ? densities_out : ws.den.as<float>(n);
        exact_mean(ws, dist, n, k, b.mean, s);
        density_from_mean(dist, n, k, o.density_kernel == FDB200_GAUSSIAN, b.mean, den, s);
        if (!o.outputs_on_device) download(densities_out, den, sizeof(float) * n, o, s);
        double m = 0.0;
        FDB_CUDA(cudaMemcpyAsync(&m, b.mean, sizeof(double), cudaMemcpyDeviceToHost, s));
        FDB_CUDA(cudaStreamSynchronize(s));
        if (mean_out) *mean_out = m;
    });
}

int fdb200_dc_detection(const int* knn_idx, const float* densities, int n, int k, const FdB200Opts* opts,
                        int* parent_out, int* cores_out, int* num_cores_out)
{
    return guarded(opts, nullptr, nullptr, [&](Workspace& ws, const FdB200Opts& o, cudaStream_t s) {
        FDB_REQUIRE(knn_idx && densities && parent_out && n > 0 && k > 0, "fdb200_dc_detection: bad arguments");
        const int* idx = upload_i32(ws.idx, knn_idx, (size_t)n * k, o, s);
        const float* den = upload_f32(ws.den, densities, (size_t)n, o, s);
        int* parent = ws.parent.as<int>(n);
        int* cores = ws.cores.as<int>(n);
        const int nc = dc_detection(ws, idx, den, n, k, parent, cores, s);
        download(parent_out, parent, sizeof(int) * n, o, s);
        download(cores_out, cores, sizeof(int) * nc, o, s);
        FDB_CUDA(cudaStreamSynchronize(s));
        if (num_cores_out) *num_cores_out = nc;
    });
}

int fdb200_final_cluster(const int* parent, int n, const int* centers, int c, const FdB200Opts* opts,
                         int* labels_out)
{
    return guarded(opts, nullptr, nullptr, [&](Workspace& ws, const FdB200Opts& o, cudaStream_t s) {
        FDB_REQUIRE(parent && labels_out && n > 0 && c >= 0 && (c == 0 || centers), "fdb200_final_cluster: bad arguments");
        const int* par = upload_i32(ws.parent, parent, (size_t)n, o, s);
        FitBuffers b = carve(ws, n, c);
        if (c > 0) {
            if (o.inputs_on_device)
                FDB_CUDA(cudaMemcpyAsync(b.centers, centers, sizeof(int) * c, cudaMemcpyDeviceToDevice, s));
            else
                FDB_CUDA(cudaMemcpyAsync(b.centers, centers, sizeof(int) * c, cudaMemcpyHostToDevice, s));
        }
        final_cluster(ws, par, n, b.centers, c, b.labels, s);
        download(labels_out, b.labels, sizeof(int) * n, o, s);
        FDB_CUDA(cudaStreamSynchronize(s));
    });
}

int fdb200_density_detection(const float* knn_dist, const int* knn_idx, int n, int k, int c, const FdB200Opts* opts,
                             float* densities_out, int* parent_out, int* cores_out, int* num_cores_out,
                             int* final_k_out)
{
    return guarded(opts, nullptr, nullptr, [&](Workspace& ws, const FdB200Opts& o, cudaStream_t s) {
        FDB_REQUIRE(knn_dist && knn_idx && densities_out && parent_out && cores_out && n >= 2 && k >= 1 && c >= 1,
                    "fdb200_density_detection: bad arguments");
        const float* dist = upload_f32(ws.dist, knn_dist, (size_t)n * k, o, s);
        const int* idx = upload_i32(ws.idx, knn_idx, (size_t)n * k, o, s);
        FitBuffers b = carve(ws, n, 1);
        float* den = o.outputs_on_device ? densities_out : ws.den.as<float>(n);
        int* parent = o.outputs_on_device ? parent_out : ws.parent.as<int>(n);
        int* cores = o.outputs_on_device ? cores_out : ws.cores.as<int>(n);
        const int gauss = (o.density_kernel == FDB200_GAUSSIAN) ? 1 : 0;
        int kk = k;
        exact_mean(ws, dist, n, kk, b.mean, s);
        density_from_mean(dist, n, kk, gauss, b.mean, den, s);
        int nc = dc_detection(ws, idx, den, n, kk, parent, cores, s);
        while (nc < c) {   // fastdecbase.cpp:186-199
            if (kk <= 1) throw Error(FDB200_ECORES, "Fit: not enough core points");
            kk /= 2;
            exact_mean(ws, dist, n, kk, b.mean, s);
            density_from_mean(dist, n, kk, gauss, b.mean, den, s);
            nc = dc_detection(ws, idx, den, n, kk, parent, cores, s);
        }
        if (!o.outputs_on_device) {
            download(densities_out, den, sizeof(float) * n, o, s);
            download(parent_out, parent, sizeof(int) * n, o, s);
            download(cores_out, cores, sizeof(int) * nc, o, s);
        }
        FDB_CUDA(cudaStreamSynchronize(s));
        if (num_cores_out) *num_cores_out = nc;
        if (final_k_out) *final_k_out = kk;
    });
}

int fdb200_dc_stage(int stage, const float* data_dev, int n, int d, const float* densities_dev, const int* cores_dev,
                    int core_nb, int p_lo, int p_hi, const FdB200Opts* opts, uint64_t* best_dev, int* rank_dev)
{
    return guarded(opts, nullptr, nullptr, [&](Workspace& ws, const FdB200Opts&, cudaStream_t s) {
        FDB_REQUIRE(stage == 0 || stage == 1, "fdb200_dc_stage: stage is 0 or 1");
        FDB_REQUIRE(data_dev && densities_dev && cores_dev && best_dev && (stage == 0 || rank_dev) && core_nb > 0 &&
                        n > 0 && d > 0 && 0 <= p_lo && p_lo <= p_hi && p_hi <= n,
                    "fdb200_dc_stage: bad arguments");
        float* norms = ws.norms.as<float>(n);
        compute_norms(data_dev, n, n, d, norms, s);
        dc_stage_range(ws, stage, data_dev, n, n, d, norms, densities_dev, cores_dev, core_nb, p_lo, p_hi, best_dev,
                       rank_dev, s);
        FDB_CUDA(cudaStreamSynchronize(s));
    });
}

int fdb200_dc_select(const float* densities_dev, const int* cores_dev, int core_nb, const uint64_t* best_dev,
                     const int* rank_dev, int num_centers, const FdB200Opts* opts, int* core_parent_dev,
                     int* centers_dev)
{
    return guarded(opts, nullptr, nullptr, [&](Workspace& ws, const FdB200Opts&, cudaStream_t s) {
        FDB_REQUIRE(densities_dev && cores_dev && best_dev && rank_dev && core_parent_dev && centers_dev &&
                        core_nb > 0 && num_centers > 0,
                    "fdb200_dc_select: bad arguments");
        dc_select(ws, densities_dev, cores_dev, core_nb, best_dev, rank_dev, num_centers, core_parent_dev, centers_dev,
                  s);
        FDB_CUDA(cudaStreamSynchronize(s));
    });
}

int fdb200_knn_partial(const float* data_dev, int n, int d, int k, const FdB200Opts* opts, uint64_t* lists_dev,
                       FdB200Stats* stats)
{
    if (stats) std::memset(stats, 0, sizeof(*stats));
    const int rc = guarded(opts, nullptr, nullptr, [&](Workspace& ws, const FdB200Opts& o, cudaStream_t s) {
        FDB_REQUIRE(data_dev && lists_dev, "fdb200_knn_partial: null pointer");
        StageTimer tm(s);
        const int a = tm.mark();
        KnnResult r = knn_lists(ws, data_dev, knn_partial_config(n, d, k, o), s);
        FDB_CUDA(cudaMemcpyAsync(lists_dev, r.lists, sizeof(uint64_t) * (size_t)n * k, cudaMemcpyDeviceToDevice, s));
        const int b = tm.mark();
        FDB_CUDA(cudaStreamSynchronize(s));
        if (stats) {
            fill_knn_stats(stats, r);
            stats->knn_ms = tm.ms(a, b);
            stats->total_ms = stats->knn_ms;
        }
    });
    if (stats) stats->launches = last_call_launches;
    return rc;
}

int fdb200_merge_lists(uint64_t* lists_dev, const uint64_t* srcs_dev, int nsrc, int n_points, int k,
                       const FdB200Opts* opts)
{
    return guarded(opts, nullptr, nullptr, [&](Workspace& ws, const FdB200Opts&, cudaStream_t s) {
        FDB_REQUIRE(lists_dev && (nsrc == 0 || srcs_dev) && n_points >= 0 && k > 0, "fdb200_merge_lists: bad arguments");
        merge_list_blocks(ws, lists_dev, srcs_dev, nsrc, n_points, k, s);
        FDB_CUDA(cudaStreamSynchronize(s));
    });
}

int fdb200_lists_to_knn(const uint64_t* lists_dev, int n, int k, const FdB200Opts* opts, float* dist_dev,
                        int* idx_dev)
{
    return guarded(opts, nullptr, nullptr, [&](Workspace&, const FdB200Opts&, cudaStream_t s) {
        FDB_REQUIRE(lists_dev && dist_dev && idx_dev && n > 0 && k > 0, "fdb200_lists_to_knn: bad arguments");
        lists_to_rank_major(lists_dev, n, k, dist_dev, idx_dev, s);
        FDB_CUDA(cudaStreamSynchronize(s));
    });
}

int fdb200_debug_tc_filter(const float* data_dev, int n, int d, const float* thr_d2_dev, const FdB200Opts* opts,
                           float* acc_dev, float* bound_dev, float* arows_dev, float* brows_dev, int* kp_out)
{
    return guarded(opts, nullptr, nullptr, [&](Workspace& ws, const FdB200Opts& o, cudaStream_t s) {
        FDB_REQUIRE(data_dev && thr_d2_dev && acc_dev && bound_dev && arows_dev && brows_dev && n >= 2 && d >= 1,
                    "fdb200_debug_tc_filter: bad arguments");
        FDB_REQUIRE(n <= 16384, "fdb200_debug_tc_filter: n is limited to 16384 (an n x n output)");
        tc_filter_audit(ws, data_dev, n, d, thr_d2_dev, o.precision, acc_dev, bound_dev, arows_dev, brows_dev, s);
        if (kp_out) *kp_out = ((d + 6 + 7) / 8) * 8;   // K of the operand rows (tc_kp)
    });
}

int fdb200_release(const FdB200Opts* opts)
{
    return guarded(opts, nullptr, nullptr, [&](Workspace& ws, const FdB200Opts&, cudaStream_t s) {
        FDB_CUDA(cudaStreamSynchronize(s));
        ws.release_all();
    });
}

}  // extern "C"
