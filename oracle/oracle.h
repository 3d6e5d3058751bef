/* oracle.h -- C API of the CPU restatement used as the parity checker.
 * Test infrastructure only: never linked into the product library. */
#ifndef OMEINSUM_ORACLE_H
#define OMEINSUM_ORACLE_H
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

#define ORC_MAX_DIMS 64
#define ORC_MAX_LABELS 4096

enum { ORC_STANDARD = 0, ORC_MAXPLUS = 1, ORC_MINPLUS = 2, ORC_MAXMUL = 3 };
enum { ORC_F32 = 0, ORC_F64 = 1 };

int orc_gemm(int alg, int dtype, const void* a, int64_t m, int64_t k, const void* b, int64_t n,
             void* c, uint32_t* argmax, int nthreads);
int orc_gemm_batched(int alg, int dtype, const void* a, int64_t batch, int64_t m, int64_t k,
                     const void* b, int64_t n, void* c, uint32_t* argmax);
int orc_copy_strided(int64_t elem_size, const void* src, int ndim, const int64_t* shape,
                     const int64_t* strides, int64_t offset, void* dst);
int orc_contract(int alg, int dtype, const void* a, int nda, const int64_t* shape_a,
                 const int64_t* strides_a, const int32_t* modes_a, const void* b, int ndb,
                 const int64_t* shape_b, const int64_t* strides_b, const int32_t* modes_b,
                 int ndc, const int64_t* shape_c, const int32_t* modes_c, void* c,
                 uint32_t* argmax);
int orc_unary(int alg, int dtype, const void* x, int nx, const int32_t* ix, const int64_t* shape_x,
              const int64_t* strides_x, int ny, const int32_t* iy, const int64_t* sizes, void* y,
              uint32_t* argmax);
int orc_max_threads(void);

#ifdef __cplusplus
}
#endif
#endif
