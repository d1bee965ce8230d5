/*
 * librouge_b200_cudnn.so: the cuDNN API subset of the reference's cuDNN
 * shim on the B200 kernels.
 *
 * The reference ships a cuDNN shim (software/rouge-numerics/include/rouge/
 * cudnn_shim.h, src/cudnn_shim.cpp) that runs the public cuDNN API on its
 * CPU code so that programs written against cuDNN run unchanged; it covers
 * convolution forward for FLOAT + NCHW only. This library exports the same
 * names with the same argument meaning, enum values and status codes, and
 * computes on the GPU: convolution forward on the sm_100a implicit-GEMM
 * tensor-core kernel (librouge_b200.so, rouge_b200_conv2d_forward) for
 * FLOAT, HALF and BFLOAT16 tensors in NCHW or NHWC, and the element-wise
 * operations as CUDA kernels.
 *
 * Memory: device pointers are used in place and the work is queued on the
 * handle's stream (asynchronous, as in cuDNN). Host pointers (the memory
 * the reference's CPU shim works on) are accepted too: such operands are
 * copied to the device and results back, and the call returns when done.
 * alpha / beta always point to host floats.
 *
 * Absent on purpose (a program that needs them fails to link instead of
 * computing something else): convolution backward, dilation, convolution
 * mode 1, DOUBLE / INT8 tensors.
 */
#pragma once

#include <driver_types.h> /* cudaStream_t */
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* cudnn_shim.h:16-28 */
typedef enum {
  CUDNN_STATUS_SUCCESS = 0,
  CUDNN_STATUS_NOT_INITIALIZED = 1,
  CUDNN_STATUS_ALLOC_FAILED = 2,
  CUDNN_STATUS_BAD_PARAM = 3,
  CUDNN_STATUS_INTERNAL_ERROR = 4,
  CUDNN_STATUS_INVALID_VALUE = 5,
  CUDNN_STATUS_ARCH_MISMATCH = 6,
  CUDNN_STATUS_MAPPING_ERROR = 7,
  CUDNN_STATUS_EXECUTION_FAILED = 8,
  CUDNN_STATUS_NOT_SUPPORTED = 9,
  CUDNN_STATUS_LICENSE_ERROR = 10
} cudnnStatus_t;

/* cudnn_shim.h:30-35, plus cuDNN's BFLOAT16 */
typedef enum {
  CUDNN_DATA_FLOAT = 0,
  CUDNN_DATA_DOUBLE = 1,
  CUDNN_DATA_HALF = 2,
  CUDNN_DATA_INT8 = 3,
  CUDNN_DATA_BFLOAT16 = 9
} cudnnDataType_t;

typedef enum { CUDNN_TENSOR_NCHW = 0, CUDNN_TENSOR_NHWC = 1 } cudnnTensorFormat_t;

/* cudnn_shim.h:39-44: every listed algorithm runs the same implicit GEMM */
typedef enum {
  CUDNN_CONVOLUTION_FWD_ALGO_IMPLICIT_GEMM = 0,
  CUDNN_CONVOLUTION_FWD_ALGO_GEMM = 2,
  CUDNN_CONVOLUTION_FWD_ALGO_DIRECT = 3,
  CUDNN_CONVOLUTION_FWD_ALGO_WINOGRAD = 6
} cudnnConvolutionFwdAlgo_t;

typedef struct rouge_b200_cudnn_ctx *cudnnHandle_t;
typedef struct rouge_b200_cudnn_tensor *cudnnTensorDescriptor_t;
typedef struct rouge_b200_cudnn_filter *cudnnFilterDescriptor_t;
typedef struct rouge_b200_cudnn_conv *cudnnConvolutionDescriptor_t;

/* cudnn_shim.h:51-54 */
const char *cudnnGetErrorString(cudnnStatus_t status);
cudnnStatus_t cudnnCreate(cudnnHandle_t *handle);
cudnnStatus_t cudnnDestroy(cudnnHandle_t handle);
size_t cudnnGetVersion(void);

/* Stream of the handle (cuDNN API; the reference's shim has none: it runs
 * on the host). NULL = the legacy default stream. */
cudnnStatus_t cudnnSetStream(cudnnHandle_t handle, cudaStream_t streamId);
cudnnStatus_t cudnnGetStream(cudnnHandle_t handle, cudaStream_t *streamId);

/* cudnn_shim.h:56-68 (cudnn_shim.cpp:83-147) */
cudnnStatus_t cudnnCreateTensorDescriptor(cudnnTensorDescriptor_t *desc);
cudnnStatus_t cudnnSetTensor4dDescriptor(cudnnTensorDescriptor_t desc, cudnnTensorFormat_t format,
                                         cudnnDataType_t type, int n, int c, int h, int w);
cudnnStatus_t cudnnDestroyTensorDescriptor(cudnnTensorDescriptor_t desc);

cudnnStatus_t cudnnCreateFilterDescriptor(cudnnFilterDescriptor_t *desc);
cudnnStatus_t cudnnSetFilter4dDescriptor(cudnnFilterDescriptor_t desc, cudnnDataType_t type,
                                         cudnnTensorFormat_t format, int k, int c, int h, int w);
cudnnStatus_t cudnnDestroyFilterDescriptor(cudnnFilterDescriptor_t desc);

/* cudnn_shim.h:70-82 (cudnn_shim.cpp:149-186): pad_h == pad_w,
 * stride_h == stride_w, dilation 1, mode 0 (cross-correlation); otherwise
 * CUDNN_STATUS_NOT_SUPPORTED. */
cudnnStatus_t cudnnCreateConvolutionDescriptor(cudnnConvolutionDescriptor_t *d);
cudnnStatus_t cudnnSetConvolution2dDescriptor(cudnnConvolutionDescriptor_t d, int pad_h, int pad_w,
                                              int stride_h, int stride_w, int dilation_h,
                                              int dilation_w, int mode, cudnnDataType_t type);
cudnnStatus_t cudnnDestroyConvolutionDescriptor(cudnnConvolutionDescriptor_t d);

cudnnStatus_t cudnnGetConvolution2dForwardOutputDim(const cudnnConvolutionDescriptor_t convDesc,
                                                    const cudnnTensorDescriptor_t inputDesc,
                                                    const cudnnFilterDescriptor_t filterDesc,
                                                    int *n, int *c, int *h, int *w);

/* cuDNN API (the reference's shim needs no workspace): bytes of device
 * workspace cudnnConvolutionForward uses for these descriptors; 0 for
 * 16-bit NHWC data with C % 64 == 0 and K % 8 == 0. */
cudnnStatus_t cudnnGetConvolutionForwardWorkspaceSize(
    cudnnHandle_t handle, const cudnnTensorDescriptor_t xDesc,
    const cudnnFilterDescriptor_t wDesc, const cudnnConvolutionDescriptor_t convDesc,
    const cudnnTensorDescriptor_t yDesc, cudnnConvolutionFwdAlgo_t algo, size_t *sizeInBytes);

/* cudnn_shim.h:84-91 (cudnn_shim.cpp:188-232): y = alpha * conv(x, w) +
 * beta * y. x, w and y of one type: FLOAT (tf32 tensor cores with split
 * operands, f32-accurate), HALF or BFLOAT16 (f32 accumulation, rounded
 * once); x / y in NCHW or NHWC each, the filter in NCHW (KCRS) or NHWC
 * (KRSC). y is read only when beta != 0. A workspace smaller than
 * cudnnGetConvolutionForwardWorkspaceSize (NULL, 0 as the reference's
 * callers pass) is replaced by one the handle owns. */
cudnnStatus_t cudnnConvolutionForward(cudnnHandle_t handle, const void *alpha,
                                      const cudnnTensorDescriptor_t xDesc, const void *x,
                                      const cudnnFilterDescriptor_t wDesc, const void *w,
                                      const cudnnConvolutionDescriptor_t convDesc,
                                      cudnnConvolutionFwdAlgo_t algo, void *workSpace,
                                      size_t workSpaceSizeInBytes, const void *beta,
                                      const cudnnTensorDescriptor_t yDesc, void *y);

/* --- Element-wise operations (cudnn_shim.h:93-178) ---------------------
 * x and y descriptors must agree in dims, type and format (NCHW or NHWC),
 * else CUDNN_STATUS_NOT_SUPPORTED. Activation and AddTensor take FLOAT,
 * HALF and BFLOAT16 (computed in f32); Softmax and BatchNorm FLOAT. */

typedef enum {
  CUDNN_ACTIVATION_SIGMOID = 0,
  CUDNN_ACTIVATION_RELU = 1,
  CUDNN_ACTIVATION_TANH = 2,
  CUDNN_ACTIVATION_CLIPPED_RELU = 3
} cudnnActivationMode_t;

typedef enum { CUDNN_NOT_PROPAGATE_NAN = 0, CUDNN_PROPAGATE_NAN = 1 } cudnnNanPropagation_t;

typedef struct rouge_b200_cudnn_act *cudnnActivationDescriptor_t;

cudnnStatus_t cudnnCreateActivationDescriptor(cudnnActivationDescriptor_t *d);
cudnnStatus_t cudnnSetActivationDescriptor(cudnnActivationDescriptor_t d,
                                           cudnnActivationMode_t mode,
                                           cudnnNanPropagation_t reluNanOpt, double coef);
cudnnStatus_t cudnnDestroyActivationDescriptor(cudnnActivationDescriptor_t d);

/* y = alpha * act(x) + beta * y (cudnn_shim.cpp:262-297); CLIPPED_RELU is
 * min(max(0, x), coef) for coef > 0, RELU otherwise. */
cudnnStatus_t cudnnActivationForward(cudnnHandle_t handle, cudnnActivationDescriptor_t actDesc,
                                     const void *alpha, const cudnnTensorDescriptor_t xDesc,
                                     const void *x, const void *beta,
                                     const cudnnTensorDescriptor_t yDesc, void *y);

/* B = alpha1 * A + alpha2 * B (cudnn_shim.cpp:299-314). A's dims equal B's
 * or are 1 (broadcast, e.g. a 1 x C x 1 x 1 bias); other shapes
 * CUDNN_STATUS_NOT_SUPPORTED. */
cudnnStatus_t cudnnAddTensor(cudnnHandle_t handle, const void *alpha1,
                             const cudnnTensorDescriptor_t aDesc, const void *A,
                             const void *alpha2, const cudnnTensorDescriptor_t bDesc, void *B);

typedef enum {
  CUDNN_SOFTMAX_FAST = 0,
  CUDNN_SOFTMAX_ACCURATE = 1,
  CUDNN_SOFTMAX_LOG = 2
} cudnnSoftmaxAlgorithm_t;

typedef enum { CUDNN_SOFTMAX_MODE_INSTANCE = 0, CUDNN_SOFTMAX_MODE_CHANNEL = 1 } cudnnSoftmaxMode_t;

/* y = alpha * softmax(x) + beta * y (cudnn_shim.cpp:316-366): INSTANCE over
 * the C*H*W values of each image, CHANNEL over C at each (n, h, w); LOG
 * gives log-softmax. */
cudnnStatus_t cudnnSoftmaxForward(cudnnHandle_t handle, cudnnSoftmaxAlgorithm_t algo,
                                  cudnnSoftmaxMode_t mode, const void *alpha,
                                  const cudnnTensorDescriptor_t xDesc, const void *x,
                                  const void *beta, const cudnnTensorDescriptor_t yDesc, void *y);

typedef enum { CUDNN_BATCHNORM_SPATIAL = 0, CUDNN_BATCHNORM_PER_ACTIVATION = 1 } cudnnBatchNormMode_t;

/* y = alpha * ((x - mean) / sqrt(var + eps) * scale + bias) + beta * y
 * (cudnn_shim.cpp:368-407), per channel; bnScaleBiasMeanVarDesc is a
 * 1 x C x 1 x 1 FLOAT descriptor of the four vectors; epsilon >= 0. */
cudnnStatus_t cudnnBatchNormalizationForwardInference(
    cudnnHandle_t handle, cudnnBatchNormMode_t mode, const void *alpha, const void *beta,
    const cudnnTensorDescriptor_t xDesc, const void *x, const cudnnTensorDescriptor_t yDesc,
    void *y, const cudnnTensorDescriptor_t bnScaleBiasMeanVarDesc, const void *scale,
    const void *bias, const void *estimatedMean, const void *estimatedVariance, double epsilon);

#ifdef __cplusplus
} /* extern "C" */
#endif
