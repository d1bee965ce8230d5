// Operand staging shared by the cuBLAS- and cuDNN-API libraries.
//
// The reference's shims are CPU libraries: their callers pass host memory.
// The B200 shims take device pointers in place (queued on the handle's
// stream, as the real libraries do) and also accept host pointers: each
// host operand of a call is copied into a device buffer the handle owns,
// the call runs on the copies, results are copied back and the call
// returns when they have arrived.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace rb200shim {

// True for memory the kernels cannot address in place: pageable host
// memory (unknown to CUDA) and page-locked host allocations.
inline bool is_host_memory(const void *p) {
  if (!p) return false;
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return true;
  }
  return a.type == cudaMemoryTypeUnregistered || a.type == cudaMemoryTypeHost;
}

// A device buffer that grows on demand (after the stream's queued work,
// which may still read the old one).
struct DevBuf {
  void *p = nullptr;
  size_t bytes = 0;
  bool ensure(size_t need, cudaStream_t st) {
    if (need <= bytes) return true;
    if (p) {
      cudaStreamSynchronize(st);
      cudaFree(p);
      p = nullptr;
      bytes = 0;
    }
    if (cudaMalloc(&p, need) != cudaSuccess) {
      cudaGetLastError();
      return false;
    }
    bytes = need;
    return true;
  }
  void release(cudaStream_t st) {
    if (p) {
      cudaStreamSynchronize(st);
      cudaFree(p);
    }
    p = nullptr;
    bytes = 0;
  }
};

// The host operands of one call. add() each operand (bytes it spans, and
// whether the call reads and / or writes it), then begin(), dev() for the
// address to compute on, and finish() after the work is queued.
class Staging {
 public:
  static constexpr int kMax = 8;
  Staging(DevBuf &buf, cudaStream_t st) : buf_(buf), st_(st) {}

  // The same pointer added twice (an in-place operation) is one operand
  // with the union of the two uses.
  void add(const void *p, size_t bytes, bool in, bool out) {
    if (!p || bytes == 0) return;
    for (int i = 0; i < n_; ++i)
      if (e_[i].host == p) {
        e_[i].in = e_[i].in || in;
        e_[i].out = e_[i].out || out;
        if (bytes > e_[i].bytes) {  // re-place it at the end with the larger size
          e_[i].bytes = bytes;
          e_[i].off = total_;
          total_ += (bytes + 255) / 256 * 256;
        }
        return;
      }
    if (n_ == kMax || !is_host_memory(p)) return;
    e_[n_++] = Entry{p, bytes, in, out, total_};
    total_ += (bytes + 255) / 256 * 256;
  }

  // Allocates the staging memory and queues the copies in.
  bool begin() {
    if (!n_) return true;
    if (!buf_.ensure(total_, st_)) return false;
    for (int i = 0; i < n_; ++i)
      if (e_[i].in && cudaMemcpyAsync(static_cast<uint8_t *>(buf_.p) + e_[i].off, e_[i].host,
                                      e_[i].bytes, cudaMemcpyHostToDevice, st_) != cudaSuccess)
        return false;
    return true;
  }

  template <class T>
  T *dev(const T *p) const {
    for (int i = 0; i < n_; ++i)
      if (e_[i].host == p)
        return reinterpret_cast<T *>(static_cast<uint8_t *>(buf_.p) + e_[i].off);
    return const_cast<T *>(p);
  }

  // Queues the copies out and waits for them (nothing to do without host
  // operands: the call stays asynchronous).
  bool finish() {
    if (!n_) return true;
    bool ok = true;
    for (int i = 0; i < n_; ++i)
      if (e_[i].out && cudaMemcpyAsync(const_cast<void *>(e_[i].host),
                                       static_cast<uint8_t *>(buf_.p) + e_[i].off, e_[i].bytes,
                                       cudaMemcpyDeviceToHost, st_) != cudaSuccess)
        ok = false;
    return cudaStreamSynchronize(st_) == cudaSuccess && ok;
  }

  bool any() const { return n_ > 0; }

 private:
  struct Entry {
    const void *host;
    size_t bytes;
    bool in, out;
    size_t off;
  };
  DevBuf &buf_;
  cudaStream_t st_;
  Entry e_[kMax];
  int n_ = 0;
  size_t total_ = 0;
};

}  // namespace rb200shim
