/* int8 GEMM int32 accumulator — C restatement (test infrastructure).
 *
 * Follows the reference kernel kernels/int8_gemm/int8_gemm.py:59-78: an exact int32 sum
 * over K of int8 x int8 products (`tl.dot(a, b, acc, out_dtype=tl.int32)`, :78).
 * B is taken either as [K,N] row-major (the reference API's layout, int8_gemm.py:100) or as
 * [N,K] row-major.  Rows of C are independent, so they are split over POSIX threads.
 */
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>

typedef struct {
  const int8_t* A;
  const int8_t* B; /* [N,K] */
  int32_t* C;
  int64_t m0, m1, N, K;
} job_t;

static void* run_rows(void* arg) {
  const job_t* j = (const job_t*)arg;
  for (int64_t m = j->m0; m < j->m1; ++m) {
    const int8_t* a = j->A + m * j->K;
    int32_t* c = j->C + m * j->N;
    for (int64_t n = 0; n < j->N; ++n) {
      const int8_t* b = j->B + n * j->K;
      int32_t acc = 0;
      for (int64_t k = 0; k < j->K; ++k) acc += (int32_t)a[k] * (int32_t)b[k];
      c[n] = acc;
    }
  }
  return 0;
}

/* C[m,n] = sum_k A[m,k] * B[n,k];  A [M,K], B [N,K], C [M,N], all row-major. */
int oracle_int8_gemm_i32_nk(const int8_t* A, const int8_t* B, int32_t* C, int64_t M, int64_t N, int64_t K,
                            int nthreads) {
  if (nthreads < 1) nthreads = 1;
  if (nthreads > 256) nthreads = 256;
  if (nthreads > M) nthreads = M > 0 ? (int)M : 1;
  pthread_t th[256];
  job_t jobs[256];
  int started = 0;
  for (int t = 0; t < nthreads; ++t) {
    jobs[t].A = A;
    jobs[t].B = B;
    jobs[t].C = C;
    jobs[t].N = N;
    jobs[t].K = K;
    jobs[t].m0 = M * t / nthreads;
    jobs[t].m1 = M * (t + 1) / nthreads;
    if (t == nthreads - 1 || pthread_create(&th[t], 0, run_rows, &jobs[t]) != 0) {
      run_rows(&jobs[t]); /* last slice (or a failed spawn) runs on the caller */
    } else {
      ++started;
    }
  }
  for (int t = 0; t < nthreads - 1; ++t)
    if (t < started) pthread_join(th[t], 0);
  return 0;
}

/* C[m,n] = sum_k A[m,k] * B[k,n];  B [K,N] row-major (transposed once into [N,K]). */
int oracle_int8_gemm_i32_kn(const int8_t* A, const int8_t* B, int32_t* C, int64_t M, int64_t N, int64_t K,
                            int nthreads) {
  int8_t* bt = (int8_t*)malloc((size_t)(N * K > 0 ? N * K : 1));
  if (!bt) return 1;
  for (int64_t k = 0; k < K; ++k)
    for (int64_t n = 0; n < N; ++n) bt[n * K + k] = B[k * N + n];
  int r = oracle_int8_gemm_i32_nk(A, bt, C, M, N, K, nthreads);
  free(bt);
  return r;
}
