/*
 * vlak_comparators.h -- C ABI of the library comparators for the row softmax
 * (libvlak_comparators.so). These are benchmark bars, not the product path:
 * the vendor softmax of cuDNN and a block-per-row softmax on CUB's
 * BlockReduce, as the reference's comparator extension provides them
 * (kernels/softmax/softmax_baselines.cu:23-55, :57-117; Python
 * softmax_cudnn / softmax_cub, kernels/softmax/__init__.py:78-114).
 *
 * Same conventions as vlak_b200.h: device pointers, a cudaStream_t passed as
 * void*, an int status (0 = ok), launches asynchronous on the stream.
 */
#ifndef VLAK_COMPARATORS_H_
#define VLAK_COMPARATORS_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define VLAK_CMP_API __attribute__((visibility("default")))
#else
#define VLAK_CMP_API
#endif

enum {
  VLAK_CMP_OK = 0,
  VLAK_CMP_ERR_INVALID_ARGUMENT = 1,
  VLAK_CMP_ERR_UNSUPPORTED_DTYPE = 3,
  VLAK_CMP_ERR_CUDA = 4,
  VLAK_CMP_ERR_CUDNN = 7
};

/* element types (the values of vlak_b200.h) */
enum { VLAK_CMP_F32 = 0, VLAK_CMP_F16 = 1, VLAK_CMP_BF16 = 2 };

/* One-line description of the last nonzero status on this thread. */
VLAK_CMP_API const char* vlak_cmp_last_error_message(void);

/* Row softmax of a contiguous [rows, cols] tensor through
 * cudnnSoftmaxForward (CUDNN_SOFTMAX_ACCURATE, instance mode over an NCHW
 * (rows, cols, 1, 1) view). Replaces softmax_cudnn
 * (kernels/softmax/softmax_baselines.cu:23-55). One cuDNN handle per device
 * and host thread, created on first use. */
VLAK_CMP_API int vlak_softmax_cudnn_fwd(const void* x, void* y, int64_t rows, int64_t cols,
                                        int dtype, void* stream);

/* Row softmax, one 256-thread block per row, max and sum through
 * cub::BlockReduce, three passes over the row, fp32 math. Replaces
 * softmax_cub (kernels/softmax/softmax_baselines.cu:57-117). */
VLAK_CMP_API int vlak_softmax_cub_fwd(const void* x, void* y, int64_t rows, int64_t cols,
                                      int dtype, void* stream);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* VLAK_COMPARATORS_H_ */
