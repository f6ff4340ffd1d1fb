// graphio.cpp -- binary files around the fit: the dataset as raw float32 (no text parsing) and the kNN
// graph, saved once so that the stages after the kNN can be re-run for other k or cluster counts.
//
// Dataset (.fbin): int32 n, int32 d, then n * d float32 row-major (one point per row), little endian --
// the binary layout of the big-ANN benchmark files. The reference reads CSV text only (get_rows_coloumns
// + read_data, helper.cpp:9-63, then the host transpose of test.cpp:110-115); this input skips the text
// parse and is transposed into the dim-major layout Fit takes by all host threads.
//
// kNN graph: a 32-byte header (magic "FDBKNNG1", uint32 version 1, int32 n, int32 k, uint32 flags,
// uint64 FNV-1a hash of the distance and index bytes), then k * n float32 distances and k * n int32
// indices, both RANK-MAJOR ([q * n + i]) exactly as compute_knn returns them (fastdecbase.h:43-46). The
// reference recomputes the graph on every Fit; its k-halving loop (fastdecbase.cpp:186-199) only ever
// reuses the first ranks of a graph in memory. A saved graph of k ranks serves any k' <= k (the first
// k' ranks of each point are its k' nearest), so sweeps over k and c need one kNN.
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "fdb_internal.h"

namespace fdb {
namespace {

constexpr char kGraphMagic[8] = {'F', 'D', 'B', 'K', 'N', 'N', 'G', '1'};
constexpr uint32_t kGraphVersion = 1;

struct GraphHeader {
    char magic[8];
    uint32_t version;
    int32_t n, k;
    uint32_t flags;
    uint64_t hash;
};
static_assert(sizeof(GraphHeader) == 32, "graph header is 32 bytes");

struct File {
    FILE* f = nullptr;
    File(const char* path, const char* mode) : f(fopen(path, mode)) {}
    ~File()
    {
        if (f) fclose(f);
    }
};

long long file_size(FILE* f)
{
    if (fseek(f, 0, SEEK_END) != 0) return -1;
    const long long sz = ftell(f);
    if (fseek(f, 0, SEEK_SET) != 0) return -1;
    return sz;
}

int host_threads(int requested)
{
    const int t = requested > 0 ? requested : (int)std::thread::hardware_concurrency();
    return std::max(1, std::min(t, 64));
}

uint64_t fnv1a(uint64_t h, const void* p, size_t bytes)
{
    const unsigned char* b = (const unsigned char*)p;
    for (size_t i = 0; i < bytes; ++i) {
        h ^= b[i];
        h *= 1099511628211ull;
    }
    return h;
}

// the hash of a graph's payload: FNV-1a over the distance bytes, then over the index bytes
uint64_t graph_hash(const float* dist, const int* idx, size_t count)
{
    uint64_t h = 1469598103934665603ull;
    h = fnv1a(h, dist, count * sizeof(float));
    return fnv1a(h, idx, count * sizeof(int));
}

template <typename Fn>
int io_guard(const char* what, Fn fn)
{
    try {
        fn();
        set_last_error("");
        return FDB200_OK;
    } catch (const Error& e) {
        set_last_error(e.what());
        return e.code;
    } catch (const std::bad_alloc&) {
        set_last_error(std::string(what) + ": host allocation failed");
        return FDB200_ENOMEM;
    } catch (const std::exception& e) {
        set_last_error(e.what());
        return FDB200_EINTERNAL;
    }
}

void read_fbin_header(FILE* f, const char* path, int& n, int& d)
{
    int32_t hdr[2] = {0, 0};
    FDB_REQUIRE(fread(hdr, sizeof(int32_t), 2, f) == 2, std::string("fbin: cannot read the header of ") + path);
    const long long sz = file_size(f);
    FDB_REQUIRE(hdr[0] > 0 && hdr[1] > 0, std::string("fbin: bad shape in ") + path);
    FDB_REQUIRE(sz == 8 + 4ll * hdr[0] * hdr[1],
                std::string(path) + " holds " + std::to_string(sz) + " bytes, but its header says " +
                    std::to_string(hdr[0]) + " x " + std::to_string(hdr[1]) + " float32 values");
    n = hdr[0];
    d = hdr[1];
}

}  // namespace
}  // namespace fdb

using namespace fdb;

extern "C" int fdb200_fbin_shape(const char* path, int* n_out, int* d_out)
{
    return io_guard("fdb200_fbin_shape", [&] {
        FDB_REQUIRE(path && n_out && d_out, "fdb200_fbin_shape: null pointer");
        File f(path, "rb");
        FDB_REQUIRE(f.f, std::string("fdb200_fbin_shape: cannot open ") + path);
        read_fbin_header(f.f, path, *n_out, *d_out);
    });
}

extern "C" int fdb200_read_fbin(const char* path, int n, int d, float* out_dim_major, int threads)
{
    return io_guard("fdb200_read_fbin", [&] {
        FDB_REQUIRE(path && out_dim_major && n > 0 && d > 0, "fdb200_read_fbin: bad arguments");
        int fn = 0, fd = 0;
        {
            File f(path, "rb");
            FDB_REQUIRE(f.f, std::string("fdb200_read_fbin: cannot open ") + path);
            read_fbin_header(f.f, path, fn, fd);
        }
        FDB_REQUIRE(fn == n && fd == d, "fdb200_read_fbin: the file is " + std::to_string(fn) + " x " +
                                            std::to_string(fd) + ", expected " + std::to_string(n) + " x " +
                                            std::to_string(d));
        // each thread reads its own rows (a separate FILE) in tiles and writes them out one dimension
        // at a time
        const int T = host_threads(threads);
        std::vector<int> fail(T, 0);
        std::vector<std::thread> pool;
        for (int t = 0; t < T; ++t)
            pool.emplace_back([&, t] {
                constexpr int kTile = 1024;
                const long long lo = (long long)n * t / T, hi = (long long)n * (t + 1) / T;
                if (lo >= hi) return;
                File f(path, "rb");
                if (!f.f || fseek(f.f, (long)(8 + 4ll * lo * d), SEEK_SET) != 0) {
                    fail[t] = 1;
                    return;
                }
                std::vector<float> tile((size_t)kTile * d);
                for (long long r0 = lo; r0 < hi; r0 += kTile) {
                    const int m = (int)std::min<long long>(kTile, hi - r0);
                    if (fread(tile.data(), sizeof(float), (size_t)m * d, f.f) != (size_t)m * d) {
                        fail[t] = 1;
                        return;
                    }
                    for (int dim = 0; dim < d; ++dim) {
                        float* o = out_dim_major + (size_t)dim * n + r0;
                        for (int q = 0; q < m; ++q) o[q] = tile[(size_t)q * d + dim];
                    }
                }
            });
        for (auto& th : pool) th.join();
        for (int v : fail) FDB_REQUIRE(!v, std::string("fdb200_read_fbin: read error in ") + path);
    });
}

extern "C" int fdb200_write_fbin(const char* path, const float* data_dim_major, int n, int d)
{
    return io_guard("fdb200_write_fbin", [&] {
        FDB_REQUIRE(path && data_dim_major && n > 0 && d > 0, "fdb200_write_fbin: bad arguments");
        File f(path, "wb");
        FDB_REQUIRE(f.f, std::string("fdb200_write_fbin: cannot create ") + path);
        const int32_t hdr[2] = {n, d};
        FDB_REQUIRE(fwrite(hdr, sizeof(int32_t), 2, f.f) == 2, "fdb200_write_fbin: write failed");
        constexpr int kTile = 1024;
        std::vector<float> tile((size_t)kTile * d);
        for (int r0 = 0; r0 < n; r0 += kTile) {
            const int m = std::min(kTile, n - r0);
            for (int dim = 0; dim < d; ++dim)
                for (int q = 0; q < m; ++q) tile[(size_t)q * d + dim] = data_dim_major[(size_t)dim * n + r0 + q];
            FDB_REQUIRE(fwrite(tile.data(), sizeof(float), (size_t)m * d, f.f) == (size_t)m * d,
                        "fdb200_write_fbin: write failed");
        }
        FDB_REQUIRE(fflush(f.f) == 0, "fdb200_write_fbin: write failed");
    });
}

extern "C" int fdb200_knn_graph_save(const char* path, const float* knn_dist, const int* knn_idx, int n, int k,
                                     int flags)
{
    return io_guard("fdb200_knn_graph_save", [&] {
        FDB_REQUIRE(path && knn_dist && knn_idx && n > 0 && k > 0, "fdb200_knn_graph_save: bad arguments");
        const size_t count = (size_t)n * k;
        GraphHeader h{};
        std::memcpy(h.magic, kGraphMagic, sizeof(h.magic));
        h.version = kGraphVersion;
        h.n = n;
        h.k = k;
        h.flags = (uint32_t)flags;
        h.hash = graph_hash(knn_dist, knn_idx, count);
        File f(path, "wb");
        FDB_REQUIRE(f.f, std::string("fdb200_knn_graph_save: cannot create ") + path);
        FDB_REQUIRE(fwrite(&h, sizeof(h), 1, f.f) == 1 && fwrite(knn_dist, sizeof(float), count, f.f) == count &&
                        fwrite(knn_idx, sizeof(int), count, f.f) == count && fflush(f.f) == 0,
                    std::string("fdb200_knn_graph_save: write failed for ") + path);
    });
}

extern "C" int fdb200_knn_graph_shape(const char* path, int* n_out, int* k_out, int* flags_out)
{
    return io_guard("fdb200_knn_graph_shape", [&] {
        FDB_REQUIRE(path && n_out && k_out, "fdb200_knn_graph_shape: null pointer");
        File f(path, "rb");
        FDB_REQUIRE(f.f, std::string("fdb200_knn_graph_shape: cannot open ") + path);
        GraphHeader h{};
        FDB_REQUIRE(fread(&h, sizeof(h), 1, f.f) == 1 && std::memcmp(h.magic, kGraphMagic, 8) == 0,
                    std::string(path) + " is not a kNN graph file");
        FDB_REQUIRE(h.version == kGraphVersion, "unsupported kNN graph file version " + std::to_string(h.version));
        FDB_REQUIRE(h.n > 0 && h.k > 0, std::string("bad shape in ") + path);
        const long long want = (long long)sizeof(h) + 8ll * h.n * h.k;
        FDB_REQUIRE(file_size(f.f) == want, std::string(path) + " is truncated or has trailing bytes");
        *n_out = h.n;
        *k_out = h.k;
        if (flags_out) *flags_out = (int)h.flags;
    });
}

extern "C" int fdb200_knn_graph_load(const char* path, int n, int k, float* knn_dist, int* knn_idx)
{
    return io_guard("fdb200_knn_graph_load", [&] {
        FDB_REQUIRE(path && knn_dist && knn_idx && n > 0 && k > 0, "fdb200_knn_graph_load: bad arguments");
        int fn = 0, fk = 0;
        if (fdb200_knn_graph_shape(path, &fn, &fk, nullptr) != FDB200_OK) throw Error(FDB200_EINVAL, fdb200_last_error());
        FDB_REQUIRE(fn == n && fk == k, "fdb200_knn_graph_load: the file holds " + std::to_string(fn) + " points x " +
                                            std::to_string(fk) + " ranks, expected " + std::to_string(n) + " x " +
                                            std::to_string(k));
        File f(path, "rb");
        FDB_REQUIRE(f.f, std::string("fdb200_knn_graph_load: cannot open ") + path);
        GraphHeader h{};
        const size_t count = (size_t)n * k;
        FDB_REQUIRE(fread(&h, sizeof(h), 1, f.f) == 1 && fread(knn_dist, sizeof(float), count, f.f) == count &&
                        fread(knn_idx, sizeof(int), count, f.f) == count,
                    std::string("fdb200_knn_graph_load: read error in ") + path);
        FDB_REQUIRE(graph_hash(knn_dist, knn_idx, count) == h.hash,
                    std::string(path) + ": the kNN graph's contents do not match its hash (corrupted file)");
        for (size_t e = 0; e < count; ++e)
            FDB_REQUIRE(knn_idx[e] >= 0 && knn_idx[e] < n, std::string(path) + ": neighbour index out of range");
    });
}
