// csv.cpp -- the reference CLI's dataset input (one point per line, comma-separated values), read in
// parallel and transposed to the dim-major layout Fit takes.
//
// The reference counts rows and columns (get_rows_coloumns, helper.cpp:9-28: every line is a row, the
// column count is the comma count of the second line + 1), parses each line with strtok + strtof on a
// single thread (read_data, helper.cpp:30-63) and then transposes on the host (test.cpp:110-115). Here
// the file is read once, cut into line-aligned byte ranges, and each thread parses its rows with
// std::from_chars (correctly rounded to nearest, like strtof) straight into the dim-major output.
#include <algorithm>
#include <charconv>
#include <cstdio>
#include <cstring>
#include <string>
#include <system_error>
#include <thread>
#include <vector>

#include "fdb_internal.h"

namespace fdb {
namespace {

struct FileBytes {
    std::vector<char> data;
    bool ok = false;
};

FileBytes slurp(const char* path)
{
    FileBytes fb;
    FILE* f = fopen(path, "rb");
    if (!f) return fb;
    if (fseek(f, 0, SEEK_END) == 0) {
        const long sz = ftell(f);
        if (sz >= 0 && fseek(f, 0, SEEK_SET) == 0) {
            fb.data.resize((size_t)sz);
            fb.ok = sz == 0 || fread(fb.data.data(), 1, (size_t)sz, f) == (size_t)sz;
        }
    }
    fclose(f);
    return fb;
}

bool blank(const char* b, const char* e)
{
    for (; b < e; ++b)
        if (*b != ' ' && *b != '\t' && *b != '\r' && *b != '\n') return false;
    return true;
}

// parse one line of comma-separated floats into out[t * n + row] for t < d; returns the count read
int parse_line(const char* b, const char* e, float* out, int n, int row, int d)
{
    int t = 0;
    const char* p = b;
    while (p < e) {
        while (p < e && (*p == ' ' || *p == '\t' || *p == '+')) ++p;   // strtof skips these too
        if (p >= e || *p == '\r' || *p == '\n') break;
        float v = 0.0f;
        const auto r = std::from_chars(p, e, v);
        if (r.ec != std::errc() && r.ec != std::errc::result_out_of_range) return -1;
        if (t < d) out[(size_t)t * n + row] = v;
        ++t;
        p = r.ptr;
        while (p < e && *p != ',') {
            if (*p != ' ' && *p != '\t' && *p != '\r' && *p != '\n') return -1;
            ++p;
        }
        if (p < e) ++p;   // the comma
    }
    return t;
}

int nthreads(int requested)
{
    int t = requested > 0 ? requested : (int)std::thread::hardware_concurrency();
    return std::max(1, std::min(t, 64));
}

// line start offsets of the file (a trailing line without a newline counts)
std::vector<size_t> line_starts(const std::vector<char>& buf, int threads)
{
    const size_t sz = buf.size();
    const int T = nthreads(threads);
    std::vector<std::vector<size_t>> part(T);
    std::vector<std::thread> pool;
    for (int t = 0; t < T; ++t)
        pool.emplace_back([&, t] {
            const size_t lo = sz * t / T, hi = sz * (t + 1) / T;
            for (size_t i = lo; i < hi; ++i)
                if (buf[i] == '\n') part[t].push_back(i + 1);
        });
    for (auto& th : pool) th.join();
    std::vector<size_t> starts;
    if (sz > 0) starts.push_back(0);
    for (auto& v : part)
        for (size_t s : v)
            if (s < sz) starts.push_back(s);
    return starts;
}

}  // namespace
}  // namespace fdb

extern "C" int fdb200_csv_shape(const char* path, int* n_out, int* d_out)
{
    using namespace fdb;
    try {
        FDB_REQUIRE(path && n_out && d_out, "fdb200_csv_shape: null pointer");
        FileBytes fb = slurp(path);
        FDB_REQUIRE(fb.ok, std::string("fdb200_csv_shape: cannot read ") + path);
        const std::vector<size_t> st = line_starts(fb.data, 0);
        // rows: non-blank lines; columns: values on the first non-blank line
        long long rows = 0;
        int cols = -1;
        for (size_t li = 0; li < st.size(); ++li) {
            const char* b = fb.data.data() + st[li];
            const char* e = fb.data.data() + (li + 1 < st.size() ? st[li + 1] - 1 : fb.data.size());
            if (blank(b, e)) continue;
            ++rows;
            if (cols < 0) {
                float dummy = 0.0f;
                cols = parse_line(b, e, &dummy, 1, 0, 0);
                FDB_REQUIRE(cols > 0, "fdb200_csv_shape: line " + std::to_string(li + 1) + " is not a list of numbers");
            }
        }
        FDB_REQUIRE(rows > 0, std::string("fdb200_csv_shape: no data in ") + path);
        FDB_REQUIRE(rows <= 0x7fffffffLL, "fdb200_csv_shape: too many rows");
        *n_out = (int)rows;
        *d_out = cols;
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

extern "C" int fdb200_read_csv(const char* path, int n, int d, float* out_dim_major, int threads)
{
    using namespace fdb;
    try {
        FDB_REQUIRE(path && out_dim_major && n > 0 && d > 0, "fdb200_read_csv: bad arguments");
        FileBytes fb = slurp(path);
        FDB_REQUIRE(fb.ok, std::string("fdb200_read_csv: cannot read ") + path);
        const std::vector<size_t> st = line_starts(fb.data, threads);
        // non-blank lines in order; row r is the r-th of them
        std::vector<size_t> rows;
        rows.reserve(st.size());
        for (size_t li = 0; li < st.size(); ++li) {
            const char* b = fb.data.data() + st[li];
            const char* e = fb.data.data() + (li + 1 < st.size() ? st[li + 1] - 1 : fb.data.size());
            if (!blank(b, e)) rows.push_back(li);
        }
        FDB_REQUIRE((long long)rows.size() == n, "fdb200_read_csv: the file has " + std::to_string(rows.size()) +
                                                     " rows, expected " + std::to_string(n));
        const int T = nthreads(threads);
        std::vector<long long> bad(T, -1);
        std::vector<std::thread> pool;
        for (int t = 0; t < T; ++t)
            pool.emplace_back([&, t] {
                // rows are parsed into a small point-major tile, which is then written out one
                // dimension at a time: contiguous stores instead of d scattered ones per row
                constexpr int kTile = 256;
                std::vector<float> tile((size_t)kTile * d);
                const size_t lo = rows.size() * t / T, hi = rows.size() * (t + 1) / T;
                for (size_t r0 = lo; r0 < hi; r0 += kTile) {
                    const int m = (int)std::min<size_t>(kTile, hi - r0);
                    for (int q = 0; q < m; ++q) {
                        const size_t li = rows[r0 + q];
                        const char* b = fb.data.data() + st[li];
                        const char* e = fb.data.data() + (li + 1 < st.size() ? st[li + 1] - 1 : fb.data.size());
                        if (parse_line(b, e, tile.data(), kTile, q, d) != d) {
                            bad[t] = (long long)li;
                            return;
                        }
                    }
                    for (int dim = 0; dim < d; ++dim)
                        std::memcpy(out_dim_major + (size_t)dim * n + r0, tile.data() + (size_t)dim * kTile,
                                    sizeof(float) * m);
                }
            });
        for (auto& th : pool) th.join();
        for (long long li : bad)
            FDB_REQUIRE(li < 0, "fdb200_read_csv: line " + std::to_string(li + 1) + " does not hold " +
                                    std::to_string(d) + " numbers");
        set_last_error("");
        return FDB200_OK;
    } catch (const Error& e) {
        set_last_error(e.what());
        return e.code;
    } catch (const std::bad_alloc&) {
        set_last_error("fdb200_read_csv: host allocation failed");
        return FDB200_ENOMEM;
    } catch (const std::exception& e) {
        set_last_error(e.what());
        return FDB200_EINTERNAL;
    }
}

extern "C" int fdb200_write_csv(const char* path, const float* data_dim_major, int n, int d, int threads)
{
    using namespace fdb;
    try {
        FDB_REQUIRE(path && data_dim_major && n > 0 && d > 0, "fdb200_write_csv: bad arguments");
        // each thread formats a contiguous range of rows (shortest text that reads back as the same
        // float, std::to_chars), then the ranges are written in order
        const int T = nthreads(threads);
        std::vector<std::string> part(T);
        std::vector<std::thread> pool;
        for (int t = 0; t < T; ++t)
            pool.emplace_back([&, t] {
                const long long lo = (long long)n * t / T, hi = (long long)n * (t + 1) / T;
                std::string& out = part[t];
                out.reserve((size_t)(hi - lo) * d * 12);
                char buf[64];
                for (long long i = lo; i < hi; ++i) {
                    for (int k = 0; k < d; ++k) {
                        const auto r = std::to_chars(buf, buf + sizeof(buf), data_dim_major[(size_t)k * n + i]);
                        out.append(buf, r.ptr);
                        out.push_back(k + 1 < d ? ',' : '\n');
                    }
                }
            });
        for (auto& th : pool) th.join();
        FILE* f = fopen(path, "wb");
        FDB_REQUIRE(f, std::string("fdb200_write_csv: cannot create ") + path);
        bool ok = true;
        for (const std::string& s : part) ok = ok && fwrite(s.data(), 1, s.size(), f) == s.size();
        ok = (fclose(f) == 0) && ok;
        FDB_REQUIRE(ok, std::string("fdb200_write_csv: write failed for ") + path);
        set_last_error("");
        return FDB200_OK;
    } catch (const Error& e) {
        set_last_error(e.what());
        return e.code;
    } catch (const std::bad_alloc&) {
        set_last_error("fdb200_write_csv: host allocation failed");
        return FDB200_ENOMEM;
    } catch (const std::exception& e) {
        set_last_error(e.what());
        return FDB200_EINTERNAL;
    }
}
