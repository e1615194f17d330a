/* TEST INFRASTRUCTURE ONLY: a pthread twin of the reference's Go threading shell, linked with the
 * reference's own unmodified C kernels (GoKernels/ffi/matmul_{avx,scalar,dispatch}.c, compiled where
 * they lie by oracle/Makefile into oracle/_ref/). It stands in for the reference's Go FFI backend on
 * this image, which has no Go toolchain.
 *
 * Mirrors GoKernels/ffi/matmul.go: FanOutRows (:132-163, one worker per core, ranges snapped up to
 * RowBlock=8), TransposeBt (:174-214, single-threaded here: it is not on the measured decode path) and
 * the MatMulF32/NTF32/TNF32 entry points (:218-395). */
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

void MatMulRowsKernel(const double* A, const double* BT, double* O, int RowStart, int RowEnd, int K, int N, int Acc);
void MatMulTnKernel(const double* A, const double* DOut, double* DB, int PStart, int PEnd, int M, int K, int N, int Acc);
void MatMulRowsKernelF32(const float* A, const float* BT, float* O, int RowStart, int RowEnd, int K, int N, int Acc);
void MatMulTnKernelF32(const float* A, const float* DOut, float* DB, int PStart, int PEnd, int M, int K, int N, int Acc);
int CpuHasAvx2Fma(void);

enum { kRowBlock = 8 };

typedef struct RowJob {
  const void* a;
  const void* bt;
  void* out;
  int start, end, k, n, acc, f32;
} RowJob;

static void* RowWorker(void* arg) {
  RowJob* j = (RowJob*)arg;
  if (j->f32)
    MatMulRowsKernelF32((const float*)j->a, (const float*)j->bt, (float*)j->out, j->start, j->end, j->k, j->n, j->acc);
  else
    MatMulRowsKernel((const double*)j->a, (const double*)j->bt, (double*)j->out, j->start, j->end, j->k, j->n, j->acc);
  return NULL;
}

/* FanOutRows, matmul.go:132-163. */
static void FanOutRows(const void* a, const void* bt, void* out, int M, int K, int N, int acc, int f32, int workers) {
  if (workers > M) workers = M;
  if (workers < 1) workers = 1;
  int per = (M + workers - 1) / workers;
  per = ((per + kRowBlock - 1) / kRowBlock) * kRowBlock;
  if (per >= M) {
    RowJob j = {a, bt, out, 0, M, K, N, acc, f32};
    RowWorker(&j);
    return;
  }
  int cnt = (M + per - 1) / per;
  pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)cnt);
  RowJob* jobs = (RowJob*)malloc(sizeof(RowJob) * (size_t)cnt);
  for (int w = 0; w < cnt; w++) {
    int s = w * per, e = s + per < M ? s + per : M;
    jobs[w] = (RowJob){a, bt, out, s, e, K, N, acc, f32};
    pthread_create(&th[w], NULL, RowWorker, &jobs[w]);
  }
  for (int w = 0; w < cnt; w++) pthread_join(th[w], NULL);
  free(th);
  free(jobs);
}

/* MatMulNTF32, matmul.go:350-353. */
void RefMatMulNTF32(const float* a, const float* bt, float* out, int m, int k, int n, int acc, int workers) {
  FanOutRows(a, bt, out, m, k, n, acc, 1, workers);
}

/* MatMulNTF64, matmul.go:242-245. */
void RefMatMulNTF64(const double* a, const double* bt, double* out, int m, int k, int n, int acc, int workers) {
  FanOutRows(a, bt, out, m, k, n, acc, 0, workers);
}

/* MatMulF32 / MatMulF64, matmul.go:218-235,329-346: transpose b to bt, then the row kernel. */
void RefMatMulF32(const float* a, const float* b, float* out, int m, int k, int n, int workers) {
  float* bt = (float*)malloc(sizeof(float) * (size_t)n * k);
  for (int j = 0; j < n; j++)
    for (int p = 0; p < k; p++) bt[(size_t)j * k + p] = b[(size_t)p * n + j];
  FanOutRows(a, bt, out, m, k, n, 0, 1, workers);
  free(bt);
}

void RefMatMulF64(const double* a, const double* b, double* out, int m, int k, int n, int workers) {
  double* bt = (double*)malloc(sizeof(double) * (size_t)n * k);
  for (int j = 0; j < n; j++)
    for (int p = 0; p < k; p++) bt[(size_t)j * k + p] = b[(size_t)p * n + j];
  FanOutRows(a, bt, out, m, k, n, 0, 0, workers);
  free(bt);
}

/* MatMulTNF32 / MatMulTNF64 (matmul.go:252-289,358-395) on one thread. */
void RefMatMulTNF32(const float* a, const float* dout, float* db, int m, int k, int n, int acc) {
  MatMulTnKernelF32(a, dout, db, 0, k, m, k, n, acc);
}

void RefMatMulTNF64(const double* a, const double* dout, double* db, int m, int k, int n, int acc) {
  MatMulTnKernel(a, dout, db, 0, k, m, k, n, acc);
}

int RefCpuHasAvx2Fma(void) { return CpuHasAvx2Fma(); }
