/*
 * fastdec_oracle.h -- CPU restatement of the FastDEC fit, used ONLY as a test oracle.
 *
 * TEST INFRASTRUCTURE: only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
 * reference leg may load this library. The product (libfastdec_b200.so) never links it.
 *
 * Semantics restated (paths are inside the reference project cyberbull66/symwarp-fastdec):
 *   - squared norms: sequential fmaf chain over d = 0..D-1           symtriknncuda.cu:56-72
 *   - pair distance d2 = max((n_i + n_j) + (-2 * dot), 0), dot = fmaf
 *     chain over d = 0..D-1 starting from 0 (the FDS tile)           symtriknnfds.h:23-26,114-116
 *   - top-k = lexicographic (d2, index) k-smallest, self excluded;
 *     heap with strict admission, ascending candidate order         symtriknncuda.cu:104-136,183-199
 *   - final order ascending (d2, index), then sqrtf(max(d2,0))      symtriknnsort.h:13-25, symtriknncuda.cu:225-234
 *   - output rank-major: element (point i, rank q) at [q * n + i]   symtriknncuda.cu:236-251,589-599
 *   - mean kNN distance: sequential double sum, point-major order   fastdecbase.cpp:257-274
 *   - density (Laplacian / Gaussian): double exp-sum per point      fastdecbase.cpp:57-94
 *   - DC detection: first denser neighbour in rank order            fastdecbase.cpp:303-333
 *   - DC reduction: nearest strictly-denser point over all N (lex
 *     min of (d2, index)), rank = #points with d2 < d2_parent        dcreductioncuda.cu:63-187
 *   - center scoring: greedy argmax of normalised rho*delta*rank     dcreductioncuda.cu:548-619
 *   - final clustering in density-descending order                   fastdecbase.cpp:358-402
 *   - Fit stage order with the k-halving retry                       fastdecbase.cpp:159-228
 *
 * The reference computes the DC-reduction dot products with cuBLAS SGEMM (closed-source
 * summation order); this restatement uses the same fmaf chain as the kNN tiles.
 */
#ifndef FASTDEC_ORACLE_H
#define FASTDEC_ORACLE_H

#ifdef __cplusplus
extern "C" {
#endif

/* squared norms of the n points of a dim-major (d rows x n columns) matrix */
void or_norms(const float* x_dm, int n, int d, float* norms);

/* d2 of one pair, exactly as the reference FDS tile computes it */
float or_pair_d2(const float* x_dm, int n, int d, const float* norms, int i, int j);
/* every ordered pair's d2 into out[i * n + j] (test support, small n) */
void or_pair_d2_all(const float* x_dm, int n, int d, float* out);

/* full exact self-kNN; outputs rank-major sqrt'd distances and indices (k * n each).
   Returns 0 on success, -1 on bad arguments (k >= n etc.). */
int or_knn(const float* x_dm, int n, int d, int k, int threads, float* dist_rm, int* idx_rm);

/* exact kNN for a subset of rows; outputs row-major (nrows x k) squared distances and indices,
   ascending (d2, index). */
int or_knn_rows(const float* x_dm, int n, int d, int k, const int* rows, int nrows, int threads,
                float* d2_out, int* idx_out);

/* sequential double mean of the first k ranks of a rank-major list (fastdecbase.cpp:257-274) */
double or_mean_knn_dist(const float* dist_rm, int n, int k);

/* density of every point from the first k ranks; gaussian != 0 selects the Gaussian kernel */
void or_density(const float* dist_rm, int n, int k, int gaussian, float* den);

/* parent[i] = first neighbour j (rank order, first k ranks) with den[i] < den[j], else -1.
   cores receives the indices with parent -1 in ascending order; returns their count. */
int or_dc_detection(const int* idx_rm, const float* den, int n, int k, int* parent, int* cores);

/* DC reduction for the given cores; outputs per-core parent (-1 if none), delta, rank, and the
   selected centers (num_centers entries, -1 padded). Returns 0 on success. */
int or_dc_reduction(const float* x_dm, int n, int d, const float* den, const int* core_idx,
                    int core_nb, int num_centers, int threads, int* core_parent, float* delta,
                    int* rank, int* centers);

/* greedy center selection from per-core (density, delta, rank) (dcreductioncuda.cu:548-619) */
void or_select_centers(const float* core_den, const float* delta, const int* rank,
                       const int* core_idx, int core_nb, int num_centers, int* centers);

/* labels from parents (-1 = root) and centers, visiting points by density descending */
void or_final_cluster(const float* den, const int* parent, int n, const int* centers, int c,
                      int* labels);

/* the whole fit. Returns 0 on success, -1 on bad arguments, -2 when there are not enough
   cores even at k = 1 (the reference throws "Fit: not enough core points"). */
int or_fit(const float* x_dm, int n, int d, int k, int c, int gaussian, int threads,
           int* centers, int* labels, int* final_k, int* num_cores);

#ifdef __cplusplus
}
#endif

#endif
