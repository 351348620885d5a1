// TEST INFRASTRUCTURE ONLY.
//
// The standard CBLAS interface, reduced to the four routines the reference
// CPU server's BLAS adapter calls (sgemm, sger, sgemv, sasum), forwarded to
// the OpenBLAS library that numpy ships (numpy.libs/libscipy_openblas64_*.so:
// 64-bit integers, symbols prefixed "scipy_" and suffixed "64_"). This image
// has no system CBLAS; with this header on the include path the reference
// CPU server builds with its own CPDE_CPU_CBLAS option against a tuned,
// multithreaded BLAS (oracle/Makefile, target cpde_ref_cpu_server_blas).
#pragma once
#include <stdint.h>

enum CBLAS_ORDER { CblasRowMajor = 101, CblasColMajor = 102 };
enum CBLAS_TRANSPOSE { CblasNoTrans = 111, CblasTrans = 112, CblasConjTrans = 113 };

extern "C" {
void scipy_cblas_sgemm64_(int order, int transa, int transb, int64_t m, int64_t n, int64_t k, float alpha,
                          const float* a, int64_t lda, const float* b, int64_t ldb, float beta, float* c,
                          int64_t ldc);
void scipy_cblas_sger64_(int order, int64_t m, int64_t n, float alpha, const float* x, int64_t incx,
                         const float* y, int64_t incy, float* a, int64_t lda);
void scipy_cblas_sgemv64_(int order, int trans, int64_t m, int64_t n, float alpha, const float* a, int64_t lda,
                          const float* x, int64_t incx, float beta, float* y, int64_t incy);
float scipy_cblas_sasum64_(int64_t n, const float* x, int64_t incx);
}

inline void cblas_sgemm(CBLAS_ORDER order, CBLAS_TRANSPOSE transa, CBLAS_TRANSPOSE transb, int m, int n, int k,
                        float alpha, const float* a, int lda, const float* b, int ldb, float beta, float* c,
                        int ldc) {
    scipy_cblas_sgemm64_(order, transa, transb, m, n, k, alpha, a, lda, b, ldb, beta, c, ldc);
}
inline void cblas_sger(CBLAS_ORDER order, int m, int n, float alpha, const float* x, int incx, const float* y,
                       int incy, float* a, int lda) {
    scipy_cblas_sger64_(order, m, n, alpha, x, incx, y, incy, a, lda);
}
inline void cblas_sgemv(CBLAS_ORDER order, CBLAS_TRANSPOSE trans, int m, int n, float alpha, const float* a, int lda,
                        const float* x, int incx, float beta, float* y, int incy) {
    scipy_cblas_sgemv64_(order, trans, m, n, alpha, a, lda, x, incx, beta, y, incy);
}
inline float cblas_sasum(int n, const float* x, int incx) { return scipy_cblas_sasum64_(n, x, incx); }
