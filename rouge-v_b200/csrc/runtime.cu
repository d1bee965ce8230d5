// Host-side plumbing: see runtime.cuh.
#include "runtime.cuh"

#include <cudaTypedefs.h>

#include "ptx.cuh"

#include <array>
#include <atomic>

namespace rb200 {
namespace {

thread_local int g_last_error = ROUGE_B200_OK;
constexpr int kMaxDevices = 64;

struct DeviceState {
  std::once_flag probe_once;
  int status = ROUGE_B200_ENODEV;
  int sm_count = 0;
  std::once_flag err_once;
  int *err_word = nullptr;
  std::once_flag ctx_once;
  HostCallContext ctx;
};

std::array<DeviceState, kMaxDevices> &devices() {
  static std::array<DeviceState, kMaxDevices> d;
  return d;
}

int current_device_index(int *dev) {
  cudaError_t e = cudaGetDevice(dev);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return ROUGE_B200_ENODEV;
  }
  if (*dev < 0 || *dev >= kMaxDevices) return ROUGE_B200_ENODEV;
  return ROUGE_B200_OK;
}

PFN_cuTensorMapEncodeTiled_v12000 encode_tiled_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
      cudaGetLastError();
      p = nullptr;
    }
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }();
  return fn;
}

PFN_cuTensorMapEncodeIm2col_v12000 encode_im2col_fn() {
  static PFN_cuTensorMapEncodeIm2col_v12000 fn = [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeIm2col", &p, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
      cudaGetLastError();
      p = nullptr;
    }
    return reinterpret_cast<PFN_cuTensorMapEncodeIm2col_v12000>(p);
  }();
  return fn;
}

}  // namespace

int make_tmap_im2col_nhwc(CUtensorMap *tm, const void *x, CUtensorMapDataType dt, int esize, int n,
                          int h, int w, int c, int lower_w, int lower_h, int upper_w, int upper_h,
                          int channels, int pixels, int stride_w, int stride_h) {
  auto fn = encode_im2col_fn();
  if (!fn) return set_status(ROUGE_B200_ENODEV);
  if (reinterpret_cast<uintptr_t>(x) & 15u) return set_status(ROUGE_B200_EUNSUPPORTED);
  const cuuint64_t cb = static_cast<cuuint64_t>(c) * esize;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(c), static_cast<cuuint64_t>(w),
                        static_cast<cuuint64_t>(h), static_cast<cuuint64_t>(n)};
  cuuint64_t strides[3] = {cb, cb * w, cb * w * h};
  int lower[2] = {lower_w, lower_h};
  int upper[2] = {upper_w, upper_h};
  cuuint32_t estr[4] = {1, static_cast<cuuint32_t>(stride_w), static_cast<cuuint32_t>(stride_h), 1};
  CUresult r = fn(tm, dt, 4, const_cast<void *>(x), dims, strides, lower, upper,
                  static_cast<cuuint32_t>(channels), static_cast<cuuint32_t>(pixels), estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? ROUGE_B200_OK : set_status(ROUGE_B200_EUNSUPPORTED);
}

int set_status(int status) {
  if (status != ROUGE_B200_OK) g_last_error = status;
  return status;
}

int cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return ROUGE_B200_OK;
  cudaGetLastError();
  if (e == cudaErrorMemoryAllocation) return set_status(ROUGE_B200_ENOMEM);
  if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver)
    return set_status(ROUGE_B200_ENODEV);
  return set_status(ROUGE_B200_ECUDA);
}

int device_ready() {
  int dev = 0;
  if (current_device_index(&dev) != ROUGE_B200_OK) return set_status(ROUGE_B200_ENODEV);
  DeviceState &d = devices()[dev];
  std::call_once(d.probe_once, [&] {
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) {
      cudaGetLastError();
      return;
    }
    if (prop.major != 10) return;  // kernels are built for sm_100a only
    d.sm_count = prop.multiProcessorCount;
    d.status = ROUGE_B200_OK;
  });
  return d.status == ROUGE_B200_OK ? ROUGE_B200_OK : set_status(d.status);
}

namespace {
std::atomic<int> g_sm_budget{0};  // 0 = all SMs
}

int current_device() {
  int dev = 0;
  return current_device_index(&dev) == ROUGE_B200_OK ? dev : 0;
}

int current_sm_count() {
  int dev = 0;
  if (current_device_index(&dev) != ROUGE_B200_OK) return 0;
  const int n = devices()[dev].sm_count;
  const int cap = g_sm_budget.load();
  return (cap > 0 && cap < n) ? cap : n;
}

int *device_error_word() {
  int dev = 0;
  if (current_device_index(&dev) != ROUGE_B200_OK) return nullptr;
  DeviceState &d = devices()[dev];
  std::call_once(d.err_once, [&] {
    int *p = nullptr;
    if (cudaMalloc(&p, 256) != cudaSuccess) {
      cudaGetLastError();
      return;
    }
    if (cudaMemset(p, 0, 256) != cudaSuccess) {
      cudaGetLastError();
      cudaFree(p);
      return;
    }
    d.err_word = p;
  });
  return d.err_word;
}

int take_device_error(cudaStream_t stream) {
  int *w = device_error_word();
  if (!w) return set_status(ROUGE_B200_ENOMEM);
  int v = 0;
  int st = cuda_status(cudaMemcpyAsync(&v, w, sizeof(int), cudaMemcpyDeviceToHost, stream));
  if (st != ROUGE_B200_OK) return st;
  st = cuda_status(cudaStreamSynchronize(stream));
  if (st != ROUGE_B200_OK) return st;
  if (v != 0) {
    cudaMemsetAsync(w, 0, sizeof(int), stream);
    cudaStreamSynchronize(stream);
    return set_status(v);
  }
  return ROUGE_B200_OK;
}

int make_tmap_2d(CUtensorMap *tm, const void *base, CUtensorMapDataType dt, uint64_t inner,
                 uint64_t outer, uint64_t pitch_bytes, uint32_t box_inner, uint32_t box_outer,
                 CUtensorMapSwizzle swizzle) {
  auto fn = encode_tiled_fn();
  if (!fn) return set_status(ROUGE_B200_ENODEV);
  if ((reinterpret_cast<uintptr_t>(base) & 15u) || (pitch_bytes & 15u))
    return set_status(ROUGE_B200_EUNSUPPORTED);
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {pitch_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(tm, dt, 2, const_cast<void *>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? ROUGE_B200_OK : set_status(ROUGE_B200_EUNSUPPORTED);
}

HostCallContext *host_context() {
  if (device_ready() != ROUGE_B200_OK) return nullptr;
  int dev = 0;
  current_device_index(&dev);
  DeviceState &d = devices()[dev];
  std::call_once(d.ctx_once, [&] {
    cudaStream_t s[3] = {nullptr, nullptr, nullptr};
    for (auto &x : s) {
      if (cudaStreamCreateWithFlags(&x, cudaStreamNonBlocking) != cudaSuccess) {
        cudaGetLastError();
        return;
      }
    }
    for (auto &e : d.ctx.ev) {
      if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) {
        cudaGetLastError();
        return;
      }
    }
    d.ctx.in_stream = s[1];
    d.ctx.out_stream = s[2];
    d.ctx.stream = s[0];  // set last: a context with a stream is complete
  });
  if (!d.ctx.stream) {
    set_status(ROUGE_B200_ECUDA);
    return nullptr;
  }
  return &d.ctx;
}

int ensure_workspace(HostCallContext *ctx, size_t bytes) {
  if (bytes <= ctx->ws_bytes) return ROUGE_B200_OK;
  if (ctx->ws) {
    cudaStreamSynchronize(ctx->in_stream);
    cudaStreamSynchronize(ctx->stream);
    cudaStreamSynchronize(ctx->out_stream);
    cudaFree(ctx->ws);
    ctx->ws = nullptr;
    ctx->ws_bytes = 0;
  }
  size_t want = round_up(bytes, size_t(1) << 21);
  int st = cuda_status(cudaMalloc(&ctx->ws, want));
  if (st != ROUGE_B200_OK) return st;
  ctx->ws_bytes = want;
  return ROUGE_B200_OK;
}

// The wait-limit check: warp 0 waits with `limit_ns` on an mbarrier that
// nothing arrives at; when the limit passes it raises the block's abort flag
// and records ROUGE_B200_ETIMEOUT in the error word, exactly as a GEMM warp
// whose TMA or MMA partner never signals does. Warps 1-3 wait on the same
// barrier with the kernels' own limit and leave on the abort flag, so the
// launch ends after about limit_ns, not after kWaitLimitNs.
__global__ void __launch_bounds__(128) wait_limit_kernel(int *err, uint64_t limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  volatile int *abort = &abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    *abort = 0;
    mbar_init_fence();
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5;
  if (warp == 0) {
    if (!mbar_wait_for(&bar, 0, abort, limit_ns) && threadIdx.x == 0) {
      *abort = 1;
      atomicCAS(err, 0, ROUGE_B200_ETIMEOUT);
    }
  } else if (!mbar_wait(&bar, 0, abort) && (threadIdx.x & 31) == 0 && !*abort) {
    atomicCAS(err, 0, ROUGE_B200_ETIMEOUT);
  }
}

}  // namespace rb200

extern "C" {

int rouge_b200_last_error(void) { return rb200::g_last_error; }

void rouge_b200_clear_error(void) { rb200::g_last_error = ROUGE_B200_OK; }

const char *rouge_b200_status_string(int status) {
  switch (status) {
    case ROUGE_B200_OK: return "ok";
    case ROUGE_B200_EINVAL: return "invalid argument";
    case ROUGE_B200_ENODEV: return "no usable sm_100 device";
    case ROUGE_B200_ECUDA: return "CUDA runtime error";
    case ROUGE_B200_EUNSUPPORTED: return "shape or alignment not supported";
    case ROUGE_B200_ETIMEOUT: return "device-side wait timed out";
    case ROUGE_B200_ENOMEM: return "out of memory";
    case ROUGE_B200_ETOOBIG: return "problem larger than the fixed scratch area of this entry point";
    default: return "unknown status";
  }
}

const char *rouge_gemm_isa_variant(void) { return "sm_100a+tcgen05"; }

RougeGemmConfig rouge_gemm_default_config(void) {
  RougeGemmConfig c;
  c.tile_m = 64;
  c.tile_n = 64;
  c.tile_k = 32;
  c.unroll = 2;
  c.split_k = 1;
  return c;
}

int rouge_b200_device_ok(void) {
  return rb200::device_ready() == ROUGE_B200_OK ? 1 : 0;
}

/* Caps the number of SMs the persistent kernels size their grids for (0 =
 * all SMs). Leaving a few SMs free lets communication kernels that run on
 * another stream (e.g. the all-gather of the sharded GEMM) overlap. Returns
 * the previous value. */
int rouge_b200_set_sm_budget(int sms) {
  return rb200::g_sm_budget.exchange(sms > 0 ? sms : 0);
}

/* Reads and clears the device error word of the current device after
 * synchronising `stream`; returns ROUGE_B200_ETIMEOUT (or another status)
 * if a kernel reported a failure since the last call. */
int rouge_b200_sync_status(void *stream) {
  int st = rb200::device_ready();
  if (st != ROUGE_B200_OK) return st;
  return rb200::take_device_error(rb200::as_stream(stream));
}


/* Runs one CTA whose wait can never complete, bounded by limit_ns (1 ms to
 * 2 s), on `stream`: the launch ends by itself and the next
 * rouge_b200_sync_status on that stream returns ROUGE_B200_ETIMEOUT, after
 * which the context is still usable. Returns the launch status. */
int rouge_b200_check_wait_limit(unsigned long long limit_ns, void *stream) {
  int st = rb200::device_ready();
  if (st != ROUGE_B200_OK) return st;
  if (limit_ns < 1000000ull || limit_ns > 2000000000ull) return rb200::set_status(ROUGE_B200_EINVAL);
  int *err = rb200::device_error_word();
  if (!err) return rb200::set_status(ROUGE_B200_ENOMEM);
  rb200::wait_limit_kernel<<<1, 128, 0, rb200::as_stream(stream)>>>(err, limit_ns);
  return rb200::cuda_status(cudaGetLastError());
}

}  // extern "C"
