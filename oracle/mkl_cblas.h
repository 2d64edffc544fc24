/*
 * Test infrastructure (oracle): a stand-in for oneMKL's <mkl_cblas.h>, used
 * only to compile the reference's CPU path (zblas/zblas.c) into
 * oracle/_ref/ so that it can check this library's GPU results.
 *
 * The reference includes "mkl_cblas.h" (zblas/zblas.c:6) and calls fourteen
 * CBLAS routines (zblas/zblas.c:127, :141, :164, :176, :183, :189, :196,
 * :203, :299, :344, :398, :405, :411, :417, :423, :429, :435). oneMKL is not
 * installed here, so each routine forwards to numpy's bundled OpenBLAS
 * (ILP64 build, symbols `scipy_cblas_<name>64_`, 64-bit integer arguments).
 * The enum values are the ones fixed by the public CBLAS interface.
 */
#ifndef ZLIFT_ORACLE_MKL_CBLAS_H
#define ZLIFT_ORACLE_MKL_CBLAS_H
#include <stddef.h>
#include <stdint.h>

typedef enum { CblasRowMajor = 101, CblasColMajor = 102 } CBLAS_LAYOUT;
typedef CBLAS_LAYOUT CBLAS_ORDER;
typedef enum { CblasNoTrans = 111, CblasTrans = 112, CblasConjTrans = 113 } CBLAS_TRANSPOSE;

typedef int64_t zo_blasint;

void scipy_cblas_sgemm64_(CBLAS_LAYOUT, CBLAS_TRANSPOSE, CBLAS_TRANSPOSE,
                          zo_blasint, zo_blasint, zo_blasint, float,
                          const float *, zo_blasint, const float *, zo_blasint,
                          float, float *, zo_blasint);
void scipy_cblas_dgemm64_(CBLAS_LAYOUT, CBLAS_TRANSPOSE, CBLAS_TRANSPOSE,
                          zo_blasint, zo_blasint, zo_blasint, double,
                          const double *, zo_blasint, const double *, zo_blasint,
                          double, double *, zo_blasint);
void scipy_cblas_sgemv64_(CBLAS_LAYOUT, CBLAS_TRANSPOSE, zo_blasint, zo_blasint,
                          float, const float *, zo_blasint, const float *,
                          zo_blasint, float, float *, zo_blasint);
void scipy_cblas_dgemv64_(CBLAS_LAYOUT, CBLAS_TRANSPOSE, zo_blasint, zo_blasint,
                          double, const double *, zo_blasint, const double *,
                          zo_blasint, double, double *, zo_blasint);
void scipy_cblas_saxpy64_(zo_blasint, float, const float *, zo_blasint, float *, zo_blasint);
void scipy_cblas_daxpy64_(zo_blasint, double, const double *, zo_blasint, double *, zo_blasint);
void scipy_cblas_sscal64_(zo_blasint, float, float *, zo_blasint);
float scipy_cblas_sdot64_(zo_blasint, const float *, zo_blasint, const float *, zo_blasint);
double scipy_cblas_ddot64_(zo_blasint, const double *, zo_blasint, const double *, zo_blasint);
float scipy_cblas_snrm264_(zo_blasint, const float *, zo_blasint);
void scipy_cblas_scopy64_(zo_blasint, const float *, zo_blasint, float *, zo_blasint);
void scipy_cblas_sswap64_(zo_blasint, float *, zo_blasint, float *, zo_blasint);
size_t scipy_cblas_isamax64_(zo_blasint, const float *, zo_blasint);
float scipy_cblas_sasum64_(zo_blasint, const float *, zo_blasint);

#define cblas_sgemm  scipy_cblas_sgemm64_
#define cblas_dgemm  scipy_cblas_dgemm64_
#define cblas_sgemv  scipy_cblas_sgemv64_
#define cblas_dgemv  scipy_cblas_dgemv64_
#define cblas_saxpy  scipy_cblas_saxpy64_
#define cblas_daxpy  scipy_cblas_daxpy64_
#define cblas_sscal  scipy_cblas_sscal64_
#define cblas_sdot   scipy_cblas_sdot64_
#define cblas_ddot   scipy_cblas_ddot64_
#define cblas_snrm2  scipy_cblas_snrm264_
#define cblas_scopy  scipy_cblas_scopy64_
#define cblas_sswap  scipy_cblas_sswap64_
#define cblas_isamax scipy_cblas_isamax64_
#define cblas_sasum  scipy_cblas_sasum64_

#endif
