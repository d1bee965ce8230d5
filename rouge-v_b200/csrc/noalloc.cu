// rouge_gemm_i8_noalloc: the int8 GEMM drop-in (same arguments and results
// as rouge_gemm_i8) for callers that cannot let the library allocate device
// memory — a process that reserves the GPU's memory for its own allocator
// at start-up, or a loop that must not allocate once it is running.
//
// rouge_gemm_i8 stages its operands (padded to the 16-byte row pitches the
// tensor-memory loads need), the scales, the output and the kernel's status
// word in a device workspace it allocates on first use. This entry point
// stages the same data in one file-scope device array of fixed size instead,
// so it calls no cudaMalloc / cudaFree and no allocating library routine.
//
//  * Limit: the staged data must fit kNoAllocScratchBytes (64 MiB):
//    M*Kp + Kp*Np + 4*(M + N) + 4*M*N bytes plus alignment, with Kp, Np =
//    K, N rounded up to 16. Larger problems are refused with
//    ROUGE_B200_ETOOBIG before anything is copied or written.
//  * Every GPU that loads the library holds its own copy of the array until
//    the process exits.
//  * Host code sees the array's name only as a host-side stand-in, not as a
//    device address. The first call on a device (with that device current)
//    looks the device address up with cudaGetSymbolAddress and caches it
//    (only a successful lookup is cached; a failed one is retried by the
//    next call). Make that first call before any stream capture.
//  * Allocation happens once, outside the caller's loop, if the caller
//    orders it so: the array's memory is reserved by the CUDA driver when
//    it loads this file's module, and the GEMM kernel's code when it is
//    first launched. With CUDA's default lazy module loading both happen
//    during the first call on a device (and a call whose shape needs a
//    kernel variant not launched before -- 128-wide single-CTA tiles for
//    small problems, 256 x 256 CTA pairs for large ones -- loads that
//    variant's code). A caller that reserves the GPU's memory for its own
//    allocator, or enters a loop that must not allocate, makes one call of
//    each shape class it will use before that point (or runs with
//    CUDA_MODULE_LOADING=EAGER, which loads everything with the library).
//  * All calls share the array and leave their data in it. The padding and
//    the status word, which must start at zero, are cleared on every call.
//    Calls from several host threads are serialised by a lock and each call
//    synchronises before it returns; GPU work that overlapped a call's use
//    of the array would race with it.
#include <cuda_runtime.h>

#include <array>
#include <cstdint>
#include <mutex>

#include "runtime.cuh"

namespace rb200 {

int launch_gemm_i8_with_err(int M, int N, int K, const int8_t *A, long long lda, const int8_t *B,
                            long long ldb, int b_layout, const float *sa, int a_rows,
                            const float *sb, int b_cols, void *Cp, long long ldc, int out_type,
                            int *err, cudaStream_t st);

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(64) << 20;

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

struct ScratchSlot {
  std::mutex m;
  void *ptr = nullptr;  // set once a lookup succeeded
};

std::array<ScratchSlot, 64> &scratch_slots() {
  static std::array<ScratchSlot, 64> s;
  return s;
}

std::mutex &scratch_lock() {
  static std::mutex m;
  return m;
}

// Device address of the current device's copy of the array, looked up with
// that device current and cached once the lookup has succeeded. A failed
// lookup (for example the driver could not reserve the array's memory while
// loading the module) is reported and tried again on the next call.
void *scratch_for_current_device(int *status) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    cudaGetLastError();
    *status = set_status(ROUGE_B200_ENODEV);
    return nullptr;
  }
  ScratchSlot &slot = scratch_slots()[dev];
  std::lock_guard<std::mutex> g(slot.m);
  if (slot.ptr) return slot.ptr;
  void *p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e != cudaSuccess || !p) {
    cudaGetLastError();
    *status = set_status(e == cudaErrorMemoryAllocation ? ROUGE_B200_ENOMEM : ROUGE_B200_ECUDA);
    return nullptr;
  }
  slot.ptr = p;
  return p;
}

inline size_t up256(size_t b) { return round_up(b, 256); }

}  // namespace
}  // namespace rb200

using namespace rb200;

extern "C" int rouge_gemm_i8_noalloc(int M, int N, int K, const int8_t *A, const int8_t *B,
                                     const float *scales_a, int a_rows, const float *scales_b,
                                     int b_cols, float *C) {
  if (!A || !B || !scales_a || !scales_b || !C || M <= 0 || N <= 0 || K <= 0)
    return set_status(ROUGE_B200_EINVAL);
  int s = device_ready();
  if (s != ROUGE_B200_OK) return s;
  const size_t Kp = round_up(K, 16), Np = round_up(N, 16);
  const size_t na = a_rows ? M : 1, nb = b_cols ? N : 1;
  const size_t o_err = 0, o_a = 256;
  const size_t o_b = o_a + up256(M * Kp);
  const size_t o_sa = o_b + up256(Kp * Np);
  const size_t o_sb = o_sa + up256(na * 4);
  const size_t o_c = o_sb + up256(nb * 4);
  const size_t need = o_c + up256(static_cast<size_t>(M) * N * 4);
  if (need > kNoAllocScratchBytes) return set_status(ROUGE_B200_ETOOBIG);

  void *base = scratch_for_current_device(&s);
  if (!base) return s;
  uint8_t *w = static_cast<uint8_t *>(base);
  int *err = reinterpret_cast<int *>(w + o_err);
  int8_t *dA = reinterpret_cast<int8_t *>(w + o_a);
  int8_t *dB = reinterpret_cast<int8_t *>(w + o_b);
  float *dsa = reinterpret_cast<float *>(w + o_sa);
  float *dsb = reinterpret_cast<float *>(w + o_sb);
  float *dC = reinterpret_cast<float *>(w + o_c);

  std::lock_guard<std::mutex> g(scratch_lock());
  cudaStream_t st = nullptr;  // legacy default stream; the call is synchronous
  if ((s = cuda_status(cudaMemsetAsync(err, 0, sizeof(int), st))) != ROUGE_B200_OK) return s;
  if (Kp != static_cast<size_t>(K)) {  // zero K padding: it adds nothing to the sums
    if ((s = cuda_status(cudaMemsetAsync(dA, 0, M * Kp, st))) != ROUGE_B200_OK) return s;
  }
  if (Kp != static_cast<size_t>(K) || Np != static_cast<size_t>(N)) {
    if ((s = cuda_status(cudaMemsetAsync(dB, 0, Kp * Np, st))) != ROUGE_B200_OK) return s;
  }
  if ((s = cuda_status(cudaMemcpy2DAsync(dA, Kp, A, K, K, M, cudaMemcpyHostToDevice, st))) !=
      ROUGE_B200_OK)
    return s;
  if ((s = cuda_status(cudaMemcpy2DAsync(dB, Np, B, N, N, K, cudaMemcpyHostToDevice, st))) !=
      ROUGE_B200_OK)
    return s;
  if ((s = cuda_status(cudaMemcpyAsync(dsa, scales_a, na * 4, cudaMemcpyHostToDevice, st))) !=
      ROUGE_B200_OK)
    return s;
  if ((s = cuda_status(cudaMemcpyAsync(dsb, scales_b, nb * 4, cudaMemcpyHostToDevice, st))) !=
      ROUGE_B200_OK)
    return s;
  s = launch_gemm_i8_with_err(M, N, static_cast<int>(Kp), dA, static_cast<long long>(Kp), dB,
                              static_cast<long long>(Np), ROUGE_B200_B_KN, dsa, a_rows ? 1 : 0,
                              dsb, b_cols ? 1 : 0, dC, N, ROUGE_B200_OUT_F32, err, st);
  if (s != ROUGE_B200_OK) return s;
  int dev_status = 0;
  if ((s = cuda_status(cudaMemcpyAsync(&dev_status, err, sizeof(int), cudaMemcpyDeviceToHost,
                                       st))) != ROUGE_B200_OK)
    return s;
  if ((s = cuda_status(cudaStreamSynchronize(st))) != ROUGE_B200_OK) return s;
  if (dev_status != 0) return set_status(dev_status);  // C is left unwritten
  if ((s = cuda_status(cudaMemcpyAsync(C, dC, static_cast<size_t>(M) * N * 4,
                                       cudaMemcpyDeviceToHost, st))) != ROUGE_B200_OK)
    return s;
  return cuda_status(cudaStreamSynchronize(st));
}
