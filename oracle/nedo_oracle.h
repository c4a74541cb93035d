/* nedo_oracle.h -- TEST INFRASTRUCTURE ONLY: CPU restatement of the reference
 * matrix-vector path (see nedo_oracle.c for the reference file:line map). */
#ifndef NEDO_ORACLE_H
#define NEDO_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GGUF tensor type codes, include/nedo/gguf.hpp:18-19 */
enum { ORACLE_F16 = 1, ORACLE_Q4_0 = 2, ORACLE_Q8_0 = 8 };
/* summation-order flavours of the reference build */
enum { ORACLE_NATIVE = 0, ORACLE_PORTABLE = 1 };
/* status codes */
enum { ORACLE_OK = 0, ORACLE_E_TYPE = 1, ORACLE_E_ALIGN = 2, ORACLE_E_ROW = 3 };

float oracle_fp16_to_fp32(uint16_t h);
uint16_t oracle_fp32_to_fp16_rne(float f);
int oracle_row_bytes(uint32_t type, uint64_t cols, uint64_t* out);
int oracle_matvec(int flavour, uint32_t type, uint64_t rows, uint64_t cols, const void* w, const float* x, float* y);
int oracle_matvec_batch(int flavour, uint32_t type, uint64_t rows, uint64_t cols, uint64_t batch, const void* w,
                        const float* x, float* y);
int oracle_embedding_row(uint32_t type, uint64_t rows, uint64_t cols, const void* w, uint64_t row, float* out);
int oracle_abs_dot(uint32_t type, uint64_t rows, uint64_t cols, const void* w, const float* x, double* out);
int64_t oracle_argmax(const float* v, uint64_t n);

#ifdef __cplusplus
}
#endif
#endif
