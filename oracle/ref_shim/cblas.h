/* Minimal stand-in for <cblas.h>, used only to compile the reference's CPU
 * driver files so that their tiled AVX2 compute templates can be called as
 * the oracle and the timed CPU baseline.
 *
 * The reference drivers call OpenBLAS only from their comparison helpers
 * (compute_openblas / testOpenBLAS / openblas_compute), which this build never
 * calls.  The functions are therefore declared here and defined as no-ops in
 * anyoption_stub.cpp; nothing in the oracle path depends on them.
 */
#ifndef ORACLE_CBLAS_SHIM_H
#define ORACLE_CBLAS_SHIM_H

#ifdef __cplusplus
extern "C" {
#endif

enum CBLAS_ORDER { CblasRowMajor = 101, CblasColMajor = 102 };
enum CBLAS_TRANSPOSE { CblasNoTrans = 111, CblasTrans = 112, CblasConjTrans = 113 };
enum CBLAS_UPLO { CblasUpper = 121, CblasLower = 122 };
enum CBLAS_SIDE { CblasLeft = 141, CblasRight = 142 };
typedef enum CBLAS_ORDER CBLAS_LAYOUT;

void cblas_sgemm(enum CBLAS_ORDER, enum CBLAS_TRANSPOSE, enum CBLAS_TRANSPOSE, int, int, int,
                 float, const float*, int, const float*, int, float, float*, int);
void cblas_ssymm(enum CBLAS_ORDER, enum CBLAS_SIDE, enum CBLAS_UPLO, int, int, float,
                 const float*, int, const float*, int, float, float*, int);
void cblas_sscal(int, float, float*, int);
void openblas_set_num_threads(int);

#ifdef __cplusplus
}
#endif

#endif
