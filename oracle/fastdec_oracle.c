/*
 * fastdec_oracle.c -- CPU restatement of the FastDEC fit (TEST ORACLE ONLY).
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference leg may load
 * this code. Every function names the reference lines (cyberbull66/symwarp-fastdec) whose
 * behaviour it restates. Build: oracle/Makefile (gcc, -ffp-contract=off, explicit fmaf).
 */
#define _GNU_SOURCE
#include "fastdec_oracle.h"

#include <float.h>
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define OR_ROWS 16   /* rows evaluated together so each data column is streamed once per block */
#define OR_CHUNK 1024

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* (d2, index) as one unsigned key: for d2 >= 0 the float bits are monotone, so unsigned key
   order is the lexicographic (d2, index) order used by the reference heaps and sort. */
static inline uint64_t pack_key(float d2, int idx) { return ((uint64_t)f2u(d2) << 32) | (uint32_t)idx; }

/* symtriknncuda.cu:56-72 -- sequential fmaf chain from d = 0 */
void or_norms(const float* x, int n, int d, float* norms)
{
    for (int i = 0; i < n; ++i) norms[i] = 0.0f;
    for (int t = 0; t < d; ++t) {
        const float* row = x + (size_t)t * n;
        for (int i = 0; i < n; ++i) norms[i] = fmaf(row[i], row[i], norms[i]);
    }
}

/* symtriknnfds.h:23-26: fmaxf((na + nb) + (-2 * dot), 0) with two separately rounded adds */
static inline float finish_d2(float na, float nb, float dot)
{
    const float s = na + nb;             /* two separately rounded adds (-ffp-contract=off) */
    const float t = s + (-2.0f * dot);
    return fmaxf(t, 0.0f);
}

float or_pair_d2(const float* x, int n, int d, const float* norms, int i, int j)
{
    float dot = 0.0f;
    for (int t = 0; t < d; ++t) dot = fmaf(x[(size_t)t * n + i], x[(size_t)t * n + j], dot);
    return finish_d2(norms[i], norms[j], dot);
}

/* every ordered pair's d2 (out[i * n + j], the diagonal included) by the same fmaf chain and finish:
   test support for small n */
void or_pair_d2_all(const float* x, int n, int d, float* out)
{
    float* norms = (float*)malloc(sizeof(float) * (size_t)n);
    if (!norms) return;
    or_norms(x, n, d, norms);
    for (int i = 0; i < n; ++i)
        for (int j = 0; j < n; ++j) out[(size_t)i * n + j] = or_pair_d2(x, n, d, norms, i, j);
    free(norms);
}

/* ---- bounded max-heap of packed keys with strict admission (symtriknncuda.cu:104-136) ---- */
static void heap_offer(uint64_t* h, int k, uint64_t key)
{
    if (key >= h[0]) return;
    int p = 0;
    for (;;) {
        int c = 2 * p + 1;
        if (c >= k) break;
        if (c + 1 < k && h[c + 1] > h[c]) ++c;
        if (h[c] <= key) break;
        h[p] = h[c];
        p = c;
    }
    h[p] = key;
}

static int cmp_u64(const void* a, const void* b)
{
    uint64_t x = *(const uint64_t*)a, y = *(const uint64_t*)b;
    return (x > y) - (x < y);
}

typedef struct {
    const float* x; const float* norms; int n, d, k;
    const int* rows; int nrows;
    uint64_t* heaps;            /* nrows * k */
    int next;                   /* next row block, taken under the mutex */
    pthread_mutex_t mu;
} KnnJob;

static void knn_block(KnnJob* J, int b0)
{
    const int n = J->n, d = J->d, k = J->k;
    const int nr = (J->nrows - b0 < OR_ROWS) ? J->nrows - b0 : OR_ROWS;
    float xr[OR_ROWS];
    float acc[OR_ROWS][OR_CHUNK];
    int rid[OR_ROWS];
    uint64_t* heap[OR_ROWS];
    for (int r = 0; r < nr; ++r) {
        rid[r] = J->rows ? J->rows[b0 + r] : b0 + r;
        heap[r] = J->heaps + (size_t)(b0 + r) * k;
        for (int q = 0; q < k; ++q) heap[r][q] = UINT64_MAX;
    }
    for (int j0 = 0; j0 < n; j0 += OR_CHUNK) {
        const int jn = (n - j0 < OR_CHUNK) ? n - j0 : OR_CHUNK;
        for (int r = 0; r < nr; ++r) memset(acc[r], 0, sizeof(float) * (size_t)jn);
        for (int t = 0; t < d; ++t) {
            const float* col = J->x + (size_t)t * n + j0;
            for (int r = 0; r < nr; ++r) xr[r] = J->x[(size_t)t * n + rid[r]];
            for (int r = 0; r < nr; ++r) {
                const float a = xr[r];
                float* ar = acc[r];
                for (int j = 0; j < jn; ++j) ar[j] = fmaf(a, col[j], ar[j]);
            }
        }
        /* candidates arrive in ascending index order, as in the reference tile loop
           (symtriknncuda.cu:474-479); admission is the lexicographic (d2, index) test */
        for (int r = 0; r < nr; ++r) {
            const float ni = J->norms[rid[r]];
            for (int j = 0; j < jn; ++j) {
                const int g = j0 + j;
                if (g == rid[r]) continue;
                const float d2 = finish_d2(ni, J->norms[g], acc[r][j]);
                heap_offer(heap[r], k, pack_key(d2, g));
            }
        }
    }
    for (int r = 0; r < nr; ++r) qsort(heap[r], (size_t)k, sizeof(uint64_t), cmp_u64);
}

static void* knn_worker(void* arg)
{
    KnnJob* J = (KnnJob*)arg;
    for (;;) {
        pthread_mutex_lock(&J->mu);
        int b0 = J->next;
        J->next += OR_ROWS;
        pthread_mutex_unlock(&J->mu);
        if (b0 >= J->nrows) break;
        knn_block(J, b0);
    }
    return NULL;
}

static int knn_run(const float* x, int n, int d, int k, const int* rows, int nrows, int threads,
                   uint64_t* heaps)
{
    float* norms = (float*)malloc(sizeof(float) * (size_t)n);
    if (!norms) return -1;
    or_norms(x, n, d, norms);
    KnnJob J;
    J.x = x; J.norms = norms; J.n = n; J.d = d; J.k = k; J.rows = rows; J.nrows = nrows;
    J.heaps = heaps; J.next = 0;
    pthread_mutex_init(&J.mu, NULL);
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    pthread_t th[256];
    int started = 0;
    for (int t = 1; t < threads; ++t)
        if (pthread_create(&th[started], NULL, knn_worker, &J) == 0) ++started;
    knn_worker(&J);
    for (int t = 0; t < started; ++t) pthread_join(th[t], NULL);
    pthread_mutex_destroy(&J.mu);
    free(norms);
    return 0;
}

/* symtriknncuda.cu:310-633 (observable result): rank-major sqrt'd distances + indices */
int or_knn(const float* x, int n, int d, int k, int threads, float* dist_rm, int* idx_rm)
{
    if (n <= 1 || k <= 0) return 0;             /* symtriknncuda.cu:319-321 */
    if (k >= n || d <= 0) return -1;             /* symtriknncuda.cu:322-324 */
    uint64_t* heaps = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)n * k);
    if (!heaps) return -1;
    if (knn_run(x, n, d, k, NULL, n, threads, heaps) != 0) { free(heaps); return -1; }
    for (int i = 0; i < n; ++i)
        for (int q = 0; q < k; ++q) {
            uint64_t key = heaps[(size_t)i * k + q];
            dist_rm[(size_t)q * n + i] = sqrtf(fmaxf(u2f((uint32_t)(key >> 32)), 0.0f));
            idx_rm[(size_t)q * n + i] = (int)(uint32_t)key;
        }
    free(heaps);
    return 0;
}

int or_knn_rows(const float* x, int n, int d, int k, const int* rows, int nrows, int threads,
                float* d2_out, int* idx_out)
{
    if (k <= 0 || k >= n || d <= 0 || nrows < 0) return -1;
    uint64_t* heaps = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)(nrows > 0 ? nrows : 1) * k);
    if (!heaps) return -1;
    if (knn_run(x, n, d, k, rows, nrows, threads, heaps) != 0) { free(heaps); return -1; }
    for (size_t e = 0; e < (size_t)nrows * k; ++e) {
        d2_out[e] = u2f((uint32_t)(heaps[e] >> 32));
        idx_out[e] = (int)(uint32_t)heaps[e];
    }
    free(heaps);
    return 0;
}

/* fastdecbase.cpp:257-274: sequential double sum in point-major order */
double or_mean_knn_dist(const float* dist_rm, int n, int k)
{
    double m = 0.0;
    for (int i = 0; i < n; ++i)
        for (int q = 0; q < k; ++q) m += dist_rm[(size_t)q * n + i];
    return m / ((double)n * k);
}

/* fastdecbase.cpp:57-94 (range bodies) and :276-301 (mean, two_mean_sq) */
void or_density(const float* dist_rm, int n, int k, int gaussian, float* den)
{
    const double mean = or_mean_knn_dist(dist_rm, n, k);
    const double two_mean_sq = 2.0 * mean * mean;
    for (int i = 0; i < n; ++i) {
        double s = 0.0;
        for (int q = 0; q < k; ++q) {
            const float v = dist_rm[(size_t)q * n + i];
            if (gaussian) {
                const double dd = v;
                s += exp(-dd * dd / two_mean_sq);
            } else {
                const float half = -v / 2;        /* float / int: float division */
                s += exp(half / mean);
            }
        }
        den[i] = (float)s;
    }
}

/* fastdecbase.cpp:303-333 */
int or_dc_detection(const int* idx_rm, const float* den, int n, int k, int* parent, int* cores)
{
    int nc = 0;
    for (int i = 0; i < n; ++i) {
        int p = -1;
        for (int q = 0; q < k; ++q) {
            const int j = idx_rm[(size_t)q * n + i];
            if (den[i] < den[j]) { p = j; break; }
        }
        parent[i] = p;
    }
    for (int i = 0; i < n; ++i)
        if (parent[i] == -1) cores[nc++] = i;
    return nc;
}

/* dcreductioncuda.cu:548-619, restated on the host with the same float expressions */
void or_select_centers(const float* core_den, const float* g_in, const int* k_in,
                       const int* core_idx, int core_nb, int num_centers, int* centers)
{
    if (core_nb <= 0 || num_centers <= 0) return;
    float g_fill = -1.0f;
    int k_fill = -1;
    for (int i = 0; i < core_nb; ++i) {
        if (g_in[i] > g_fill) g_fill = g_in[i];
        if (k_in[i] > k_fill) k_fill = k_in[i];
    }
    float min_den = FLT_MAX, max_den = -FLT_MAX, min_g = FLT_MAX, max_g = -FLT_MAX;
    float min_k = FLT_MAX, max_k = -FLT_MAX;
    for (int i = 0; i < core_nb; ++i) {
        const float dn = core_den[i];
        const float g = (g_in[i] < 0.0f) ? g_fill : g_in[i];
        const float kk = (float)((k_in[i] < 0) ? k_fill : k_in[i]);
        if (dn < min_den) min_den = dn;
        if (dn > max_den) max_den = dn;
        if (g < min_g) min_g = g;
        if (g > max_g) max_g = g;
        if (kk < min_k) min_k = kk;
        if (kk > max_k) max_k = kk;
    }
    const float den_range = max_den - min_den;
    const float g_range = max_g - min_g;
    const float k_range = max_k - min_k;
    const int select_n = (num_centers < core_nb) ? num_centers : core_nb;
    char* chosen = (char*)calloc((size_t)core_nb, 1);
    for (int sel = 0; sel < select_n; ++sel) {
        float best_sd = -FLT_MAX;
        int best = -1;
        for (int i = 0; i < core_nb; ++i) {
            if (chosen[i]) continue;
            const float dn = core_den[i];
            const float g = (g_in[i] < 0.0f) ? g_fill : g_in[i];
            const float kk = (float)((k_in[i] < 0) ? k_fill : k_in[i]);
            const float den_n = (den_range == 0.0f) ? 1.0f : (dn - min_den) / den_range;
            const float g_n = (g_range == 0.0f) ? 1.0f : (g - min_g) / g_range;
            const float k_n = (k_range == 0.0f) ? 1.0f : (kk - min_k) / k_range;
            const float sd = den_n * g_n * k_n;
            if (sd > best_sd || (sd == best_sd && (best < 0 || i < best))) { best_sd = sd; best = i; }
        }
        centers[sel] = (best >= 0) ? core_idx[best] : -1;
        /* the reference marks a core chosen when its global index already appears among the
           selected centers (dcreductioncuda.cu:591-598); core indices are distinct */
        if (best >= 0) chosen[best] = 1;
    }
    for (int sel = select_n; sel < num_centers; ++sel) centers[sel] = -1;
    free(chosen);
}

typedef struct {
    const float* x; const float* norms; const float* den; const int* core_idx;
    int n, d, core_nb;
    int* parent; float* d2p; int* rank;
    int next;
    pthread_mutex_t mu;
} DcJob;

static void dc_one(DcJob* J, int c)
{
    const int n = J->n, d = J->d, gc = J->core_idx[c];
    const float cden = J->den[gc], cnorm = J->norms[gc];
    float* dots = (float*)malloc(sizeof(float) * (size_t)n);
    for (int j = 0; j < n; ++j) dots[j] = 0.0f;
    for (int t = 0; t < d; ++t) {
        const float a = J->x[(size_t)t * n + gc];
        const float* col = J->x + (size_t)t * n;
        for (int j = 0; j < n; ++j) dots[j] = fmaf(a, col[j], dots[j]);
    }
    /* stage A (dcreductioncuda.cu:63-111): lexicographic min over strictly denser points */
    uint64_t best = UINT64_MAX;
    for (int j = 0; j < n; ++j) {
        if (!(cden < J->den[j])) continue;
        const uint64_t key = pack_key(finish_d2(J->norms[j], cnorm, dots[j]), j);
        if (key < best) best = key;
    }
    if (best == UINT64_MAX) {
        J->parent[c] = -1; J->d2p[c] = -1.0f; J->rank[c] = -1;
    } else {
        const float d2p = u2f((uint32_t)(best >> 32));
        /* stage B (dcreductioncuda.cu:131-170): count of ALL points strictly closer */
        int cnt = 0;
        for (int j = 0; j < n; ++j)
            if (finish_d2(J->norms[j], cnorm, dots[j]) < d2p) ++cnt;
        J->parent[c] = (int)(uint32_t)best;
        J->d2p[c] = d2p;
        J->rank[c] = (cnt == 0) ? -1 : cnt;   /* dc_cb_finalize, dcreductioncuda.cu:172-187 */
    }
    free(dots);
}

static void* dc_worker(void* arg)
{
    DcJob* J = (DcJob*)arg;
    for (;;) {
        pthread_mutex_lock(&J->mu);
        int c = J->next++;
        pthread_mutex_unlock(&J->mu);
        if (c >= J->core_nb) break;
        dc_one(J, c);
    }
    return NULL;
}

/* dcreductioncuda.cu:189-545 and :621-700 */
int or_dc_reduction(const float* x, int n, int d, const float* den, const int* core_idx,
                    int core_nb, int num_centers, int threads, int* core_parent, float* delta,
                    int* rank, int* centers)
{
    if (core_nb <= 0 || num_centers <= 0 || n <= 0 || d <= 0) return -1;   /* :632-636 */
    for (int c = 0; c < core_nb; ++c)
        if (core_idx[c] < 0 || core_idx[c] >= n) return -1;                   /* :641-644 */
    float* norms = (float*)malloc(sizeof(float) * (size_t)n);
    float* d2p = (float*)malloc(sizeof(float) * (size_t)core_nb);
    float* cden = (float*)malloc(sizeof(float) * (size_t)core_nb);
    or_norms(x, n, d, norms);
    DcJob J;
    J.x = x; J.norms = norms; J.den = den; J.core_idx = core_idx; J.n = n; J.d = d;
    J.core_nb = core_nb; J.parent = core_parent; J.d2p = d2p; J.rank = rank; J.next = 0;
    pthread_mutex_init(&J.mu, NULL);
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    pthread_t th[256];
    int started = 0;
    for (int t = 1; t < threads; ++t)
        if (pthread_create(&th[started], NULL, dc_worker, &J) == 0) ++started;
    dc_worker(&J);
    for (int t = 0; t < started; ++t) pthread_join(th[t], NULL);
    pthread_mutex_destroy(&J.mu);
    for (int c = 0; c < core_nb; ++c) {
        delta[c] = (d2p[c] < 0.0f) ? -1.0f : sqrtf(d2p[c]);
        cden[c] = den[core_idx[c]];
    }
    or_select_centers(cden, delta, rank, core_idx, core_nb, num_centers, centers);
    free(norms); free(d2p); free(cden);
    return 0;
}

typedef struct { float value; int index; } ValIdx;

/* fastdecbase.h:57-64: density descending, index ascending */
static int cmp_den_desc(const void* a, const void* b)
{
    const ValIdx* fa = (const ValIdx*)a;
    const ValIdx* fb = (const ValIdx*)b;
    if (fa->value != fb->value) return (fa->value < fb->value) - (fa->value > fb->value);
    return (fa->index > fb->index) - (fa->index < fb->index);
}

/* fastdecbase.cpp:358-385 */
void or_final_cluster(const float* den, const int* parent, int n, const int* centers, int c,
                      int* labels)
{
    for (int i = 0; i < n; ++i) labels[i] = -1;
    ValIdx* v = (ValIdx*)malloc(sizeof(ValIdx) * (size_t)(n > 0 ? n : 1));
    for (int i = 0; i < n; ++i) { v[i].value = den[i]; v[i].index = i; }
    qsort(v, (size_t)n, sizeof(ValIdx), cmp_den_desc);
    for (int i = 0; i < c; ++i) labels[centers[i]] = i;
    for (int t = 0; t < n; ++t) {
        const int i = v[t].index;
        if (labels[i] == -1) labels[i] = (parent[i] == -1) ? 0 : labels[parent[i]];
    }
    free(v);
}

/* fastdecbase.cpp:159-228 */
int or_fit(const float* x, int n, int d, int k, int c, int gaussian, int threads,
           int* centers, int* labels, int* final_k, int* num_cores)
{
    if (n <= 1 || d <= 0 || k <= 0 || k >= n || c <= 0) return -1;
    float* dist = (float*)malloc(sizeof(float) * (size_t)n * k);
    int* idx = (int*)malloc(sizeof(int) * (size_t)n * k);
    float* den = (float*)malloc(sizeof(float) * (size_t)n);
    int* parent = (int*)malloc(sizeof(int) * (size_t)n);
    int* cores = (int*)malloc(sizeof(int) * (size_t)n);
    int rc = 0;
    if (or_knn(x, n, d, k, threads, dist, idx) != 0) { rc = -1; goto done; }
    {
        int kk = k;
        or_density(dist, n, kk, gaussian, den);
        int nc = or_dc_detection(idx, den, n, kk, parent, cores);
        while (nc < c) {
            if (kk <= 1) { rc = -2; goto done; }
            kk = kk / 2;   /* lists are truncated to their first kk ranks */
            or_density(dist, n, kk, gaussian, den);
            nc = or_dc_detection(idx, den, n, kk, parent, cores);
        }
        if (final_k) *final_k = kk;
        if (num_cores) *num_cores = nc;
        if (nc == c) {
            for (int i = 0; i < c; ++i) centers[i] = cores[i];
        } else {
            int* cp = (int*)malloc(sizeof(int) * (size_t)nc);
            float* dl = (float*)malloc(sizeof(float) * (size_t)nc);
            int* rk = (int*)malloc(sizeof(int) * (size_t)nc);
            rc = or_dc_reduction(x, n, d, den, cores, nc, c, threads, cp, dl, rk, centers);
            for (int i = 0; i < nc; ++i) parent[cores[i]] = cp[i];
            free(cp); free(dl); free(rk);
            if (rc != 0) goto done;
        }
        or_final_cluster(den, parent, n, centers, c, labels);
    }
done:
    free(dist); free(idx); free(den); free(parent); free(cores);
    return rc;
}
