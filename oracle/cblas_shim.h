/*
 * cblas_shim.h -- test infrastructure only (the CPU oracle build).
 *
 * The reference C executor (csrc/ops/matmul.c, csrc/ops/attn.c) calls the
 * standard CBLAS names cblas_sgemm / cblas_sgemv and links -lopenblas
 * (csrc/Makefile:12).  No system OpenBLAS or cblas.h exists in this image,
 * so the oracle build force-includes this header: it declares the standard
 * CBLAS enum values (RowMajor=101, NoTrans=111, Trans=112 -- the values the
 * CBLAS standard fixes) and maps the two entry points onto the
 * prefixed exports of the OpenBLAS that scipy bundles (scipy_cblas_*).
 */
#ifndef ORACLE_CBLAS_SHIM_H
#define ORACLE_CBLAS_SHIM_H

#ifndef __APPLE__
enum CBLAS_ORDER { CblasRowMajor = 101, CblasColMajor = 102 };
enum CBLAS_TRANSPOSE { CblasNoTrans = 111, CblasTrans = 112, CblasConjTrans = 113 };
typedef enum CBLAS_ORDER CBLAS_ORDER;
typedef enum CBLAS_TRANSPOSE CBLAS_TRANSPOSE;

void scipy_cblas_sgemm(enum CBLAS_ORDER order, enum CBLAS_TRANSPOSE ta,
                       enum CBLAS_TRANSPOSE tb, int M, int N, int K,
                       float alpha, const float* A, int lda,
                       const float* B, int ldb, float beta,
                       float* C, int ldc);
void scipy_cblas_sgemv(enum CBLAS_ORDER order, enum CBLAS_TRANSPOSE t,
                       int M, int N, float alpha, const float* A, int lda,
                       const float* x, int incx, float beta,
                       float* y, int incy);
#define cblas_sgemm scipy_cblas_sgemm
#define cblas_sgemv scipy_cblas_sgemv
#endif

#endif
