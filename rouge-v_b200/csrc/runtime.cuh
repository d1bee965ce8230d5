// Host-side plumbing shared by the launchers: status codes, device checks,
// tensor-map encoding, the per-device error word written by kernels whose
// bounded waits ran out, and the library-owned stream / workspace used by
// the host-pointer drop-in entries.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <mutex>

#include "rouge/numerics_b200.h"

namespace rb200 {

// Records `status` as this thread's last error when it is a failure.
int set_status(int status);
// Maps a CUDA runtime error to a status (ROUGE_B200_OK for cudaSuccess) and
// records it.
int cuda_status(cudaError_t e);

// ROUGE_B200_OK when the current device is a compute-capability 10.x part.
int device_ready();
// Index (below 64) of the current device; 0 if it cannot be read.
int current_device();
int current_sm_count();

// Device word (int) that kernels set to a non-zero status when a bounded
// wait gives up. One per device, allocated on first use.
int *device_error_word();
// Reads and clears the current device's error word (synchronises).
int take_device_error(cudaStream_t stream);

inline cudaStream_t as_stream(void *s) { return reinterpret_cast<cudaStream_t>(s); }

// 2-D tiled tensor map, zero fill out of bounds (128-byte swizzle unless
// another is given).
//   inner/outer: tensor extent in elements; pitch_bytes: row pitch;
//   box_inner/box_outer: box extent in elements.
int make_tmap_2d(CUtensorMap *tm, const void *base, CUtensorMapDataType dt, uint64_t inner,
                 uint64_t outer, uint64_t pitch_bytes, uint32_t box_inner, uint32_t box_outer,
                 CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B);

// 4-D im2col tensor map over NHWC activations x[n][h][w][c] (128-byte
// swizzle, zero fill): boxes of `pixels` output pixels x `channels`
// channels; lower/upper corners and traversal strides as for
// cuTensorMapEncodeIm2col.
int make_tmap_im2col_nhwc(CUtensorMap *tm, const void *x, CUtensorMapDataType dt, int esize, int n,
                          int h, int w, int c, int lower_w, int lower_h, int upper_w, int upper_h,
                          int channels, int pixels, int stride_w, int stride_h);

// Library-owned resources for the synchronous host-pointer entries, per
// device: three non-blocking streams, an event pool and a growable device
// workspace. Callers hold `lock` for the whole call. Calls that move large
// operands split them into row bands: band b's host-to-device copy runs on
// in_stream, its kernels on `stream`, its device-to-host copy on
// out_stream, so that copies in both directions and the kernels overlap;
// events from `ev` order the three per band.
constexpr int kBandEvents = 64;
struct HostCallContext {
  std::mutex lock;
  cudaStream_t stream = nullptr;
  cudaStream_t in_stream = nullptr;
  cudaStream_t out_stream = nullptr;
  cudaEvent_t ev[kBandEvents] = {};
  void *ws = nullptr;
  size_t ws_bytes = 0;
};
// Returns the context of the current device, creating the stream on first
// use; nullptr (status recorded) on failure.
HostCallContext *host_context();
// Ensures ctx->ws holds at least `bytes`; returns a status.
int ensure_workspace(HostCallContext *ctx, size_t bytes);

inline size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

}  // namespace rb200
