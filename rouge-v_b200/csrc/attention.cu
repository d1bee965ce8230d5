// Attention and the transformer block (the in-library consumers of the GEMM:
// attention.cpp:27-88, attention_gqa.cpp:52-269, transformer.cpp:33-161)
// on the tcgen05 GEMMs.
//
// Attention, per group of query heads sharing one K/V head and per block of
// query rows:
//   S = scale * Q K^T    tf32 tensor-core GEMM over split operands (3xTF32:
//                        f32-accurate scores, the reference sums in double)
//   P = softmax(S)       one warp per row, masked (causal / window / kv_off),
//                        written directly as the split A operand of the next
//   O = P V              the same GEMM, per query head, into O
// K and V are packed once per call ([hi|lo|hi] along the reduction), fp8
// caches decoded on the way (e4m3 times the head's scale, the reference's
// float product). The scores of one block are the only intermediate; blocks
// of query rows keep it within a fixed budget. Rows whose keys are all
// masked give 0, as in the reference.
//
// The transformer block chains RMSNorm, the Q/K/V projections (row-major
// 3xTF32 GEMMs on [in][out] weights), RoPE with the relayout to
// [head][token][dim], the attention, the output projection with the
// residual added in the GEMM epilogue (beta = 1 on a copy of x), RMSNorm,
// gate / up projections, SwiGLU and the down projection (again with its
// residual in the epilogue).
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <mutex>

#include "formats.cuh"
#include "pack.cuh"
#include "runtime.cuh"

extern "C" int rouge_b200_gemm_colmajor(int transa, int transb, int m, int n, int k, int ab_type,
                                        float alpha, const void *A, int lda, const void *B, int ldb,
                                        float beta, void *C, int c_type, int ldc, void *workspace,
                                        size_t workspace_bytes, void *stream);
extern "C" size_t rouge_b200_gemm_colmajor_workspace(int ab_type, int m, int n, int k);

namespace rb200 {

int launch_gemm_blas(int kind, int M, int N, int K, const void *A, long long lda, const void *B,
                     long long ldb, int b_layout, float alpha, float beta, float *Cp,
                     long long ldc, cudaStream_t st);
int launch_gemm_blas_batched(int kind, int M, int N, int K, const void *A, long long lda,
                             const void *B, long long ldb, float alpha, float beta, float *Cp,
                             long long ldc, int batch, cudaStream_t st);

namespace {

constexpr int kThreads = 256;
constexpr size_t kScoreBudget = size_t(512) << 20;  // S + split P of one query block

size_t rup(size_t v, size_t a) { return (v + a - 1) / a * a; }

unsigned grid_of(size_t items) {
  const size_t b = (items + kThreads - 1) / kThreads;
  const size_t cap = static_cast<size_t>(current_sm_count()) * 8;
  return static_cast<unsigned>(b < 1 ? 1 : (b < cap ? b : cap));
}

// e4m3 codes times a per-head scale (the reference's float product).
__global__ void decode_kv_kernel(const uint8_t *__restrict__ q, size_t per_head, int heads,
                                 const float *__restrict__ scales, float *__restrict__ out) {
  const size_t n = per_head * heads;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    out[i] = __fmul_rn(decode_e4m3(q[i]), scales[i / per_head]);
}

// Softmax rows of one query block: rows r = g * sb + i (query head g of the
// group, query s = s0 + i), scores S[r][0..Skv) with pitch lds. Keys t are
// allowed for t_lo <= t < t_hi (attention_gqa.cpp:103-112): causal: t <= s
// + kv_off; window > 0: t >= s + kv_off - window + 1. Writes P as the split
// tf32 operand [hi | hi | lo] (blocks of Kp) with zeros past Skv and at
// masked keys; an all-masked row is all zeros.
__global__ void softmax_split_kernel(const float *__restrict__ S, long long lds, int rows, int sb,
                                     int s0, int Skv, int Kp, int causal, int window, int kv_off,
                                     uint32_t *__restrict__ P) {
  const int lane = threadIdx.x & 31;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  for (int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < rows; r += warps) {
    const int s = s0 + r % sb;
    int t_lo = 0, t_hi = Skv;
    if (causal) t_hi = min(Skv, s + kv_off + 1);
    if (window > 0) t_lo = max(t_lo, s + kv_off - window + 1);
    if (t_lo < 0) t_lo = 0;
    const float *srow = S + static_cast<long long>(r) * lds;
    uint32_t *prow = P + static_cast<long long>(r) * 3 * Kp;
    float m = -INFINITY;
    for (int t = t_lo + lane; t < t_hi; t += 32) m = fmaxf(m, srow[t]);
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float sum = 0.0f;
    for (int t = t_lo + lane; t < t_hi; t += 32) sum += expf(srow[t] - m);
#pragma unroll
    for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    const bool any = t_hi > t_lo && m != -INFINITY;
    const float inv = any ? 1.0f / sum : 0.0f;
    for (int t = lane; t < Kp; t += 32) {
      const float p = (any && t >= t_lo && t < t_hi) ? expf(srow[t] - m) * inv : 0.0f;
      const float hi = tf32_round_rna(p);
      prow[t] = __float_as_uint(hi);
      prow[Kp + t] = __float_as_uint(hi);
      prow[2 * Kp + t] = __float_as_uint(p - hi);
    }
  }
}

// RMSNorm of each row (transformer.cpp:33-40): sum of squares in double,
// out = (float)(x * (1 / sqrt(ss / n + eps))) * w.
__global__ void rmsnorm_kernel(const float *__restrict__ x, int rows, int n,
                               const float *__restrict__ w, float eps, float *__restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  for (int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < rows; r += warps) {
    const float *xr = x + static_cast<size_t>(r) * n;
    double ss = 0.0;
    for (int i = lane; i < n; i += 32) ss = __fma_rn(static_cast<double>(xr[i]), xr[i], ss);
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const double inv = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(ss, n), static_cast<double>(eps))));
    float *orow = out + static_cast<size_t>(r) * n;
    for (int i = lane; i < n; i += 32)
      orow[i] = __fmul_rn(__double2float_rn(__dmul_rn(static_cast<double>(xr[i]), inv)), w[i]);
  }
}

// RoPE rotation of the pair (v[i], v[i + half]) at position pos
// (transformer.cpp:44-58): angle pos / theta^(2i / n) in double, cos and sin
// rounded to float, then x0 c - x1 s and x0 s + x1 c in float.
__device__ __forceinline__ void rope_pair(float &x0, float &x1, int i, int n, int pos, float theta) {
  const double freq = 1.0 / pow(static_cast<double>(theta), (2.0 * i) / static_cast<double>(n));
  const double a = static_cast<double>(pos) * freq;
  const float c = static_cast<float>(cos(a)), s = static_cast<float>(sin(a));
  const float a0 = x0, a1 = x1;
  x0 = __fsub_rn(__fmul_rn(a0, c), __fmul_rn(a1, s));
  x1 = __fadd_rn(__fmul_rn(a0, s), __fmul_rn(a1, c));
}

// flat [S][H * Dq] -> [H][S][Dq], RoPE at position s when rope != 0.
__global__ void relayout_rope_kernel(const float *__restrict__ flat, long long ld, int S, int H,
                                     int Dq, int rope, float theta, float *__restrict__ out) {
  const int half = Dq / 2;
  if (half == 0) rope = 0;  // (no pair to rotate: a plain relayout)
  const size_t pairs = static_cast<size_t>(S) * H * (rope ? half : Dq);
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < pairs;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    if (rope) {
      const int j = static_cast<int>(i % half);
      const size_t hs = i / half;
      const int h = static_cast<int>(hs % H), s = static_cast<int>(hs / H);
      const float *src = flat + static_cast<size_t>(s) * ld + static_cast<size_t>(h) * Dq;
      float x0 = src[j], x1 = src[j + half];
      rope_pair(x0, x1, j, Dq, s, theta);
      float *dst = out + (static_cast<size_t>(h) * S + s) * Dq;
      dst[j] = x0;
      dst[j + half] = x1;
      if ((Dq & 1) && j == 0) dst[Dq - 1] = src[Dq - 1];  // (odd Dq: the last element stays)
    } else {
      const int d = static_cast<int>(i % Dq);
      const size_t hs = i / Dq;
      const int h = static_cast<int>(hs % H), s = static_cast<int>(hs / H);
      out[(static_cast<size_t>(h) * S + s) * Dq + d] =
          flat[static_cast<size_t>(s) * ld + static_cast<size_t>(h) * Dq + d];
    }
  }
}

// [H][S][Dq] -> flat [S][H * Dq]
__global__ void unflatten_kernel(const float *__restrict__ in, int S, int H, int Dq,
                                 float *__restrict__ flat) {
  const size_t n = static_cast<size_t>(S) * H * Dq;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int d = static_cast<int>(i % Dq);
    const size_t hs = i / Dq;
    const int h = static_cast<int>(hs % H), s = static_cast<int>(hs / H);
    flat[i] = in[(static_cast<size_t>(h) * S + s) * Dq + d];
  }
}

// SwiGLU in place on gate (transformer.cpp:61-68): (g / (1 + e^-g)) * up.
__global__ void swiglu_kernel(float *__restrict__ gate, const float *__restrict__ up, size_t n) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const float g = gate[i];
    gate[i] = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), up[i]);
  }
}

// SwiGLU on the side-by-side gate | up projections gu[S][2*Dff]: the gate
// half of each row becomes silu(gate) * up, as swiglu_kernel computes it.
__global__ void swiglu_rows_kernel(float *__restrict__ gu, int S, int Dff) {
  const size_t n = static_cast<size_t>(S) * Dff;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t r = i / Dff, j = i - r * Dff;
    float *row = gu + r * 2 * Dff;
    const float g = row[j];
    row[j] = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), row[Dff + j]);
  }
}

__global__ void rope_kernel(float *x, int heads, int hd, int pos, float theta) {
  const int half = hd / 2;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < heads * half; i += gridDim.x * blockDim.x) {
    float *v = x + static_cast<size_t>(i / half) * hd;
    const int j = i % half;
    float x0 = v[j], x1 = v[j + half];
    rope_pair(x0, x1, j, hd, pos, theta);
    v[j] = x0;
    v[j + half] = x1;
  }
}

// Carves 256-byte aligned pieces from a workspace.
struct Arena {
  uint8_t *p;
  size_t used = 0, cap;
  Arena(void *base, size_t bytes) : p(static_cast<uint8_t *>(base)), cap(bytes) {}
  template <class T>
  T *take(size_t n) {
    T *r = reinterpret_cast<T *>(p + used);
    used += rup(n * sizeof(T), 256);
    return used <= cap ? r : nullptr;
  }
};

struct AttnPlan {
  int Dp, Kp, group, sb;
  // all K/V head groups at once: the sequence is one block and a group's
  // rows (group * S) a multiple of 256, so each GEMM is one batched launch
  bool all_groups;
  size_t bytes;
};

AttnPlan attn_plan(int S, int Skv, int Dh, int Hq, int Hkv, bool fp8) {
  AttnPlan a;
  a.Dp = static_cast<int>(rup(Dh, 32));
  a.Kp = static_cast<int>(rup(Skv, 32));
  a.group = Hq / Hkv;
  const size_t per_row = static_cast<size_t>(a.Kp) * 16;  // S (4 B) + split P (12 B)
  size_t sb = kScoreBudget / (per_row * a.group);
  if (sb < 16) sb = 16;
  a.sb = static_cast<int>(sb < static_cast<size_t>(S) ? sb : S);
  a.all_groups = a.sb == S && (static_cast<size_t>(a.group) * S) % 256 == 0 && Hkv > 1 &&
                 static_cast<size_t>(Hkv) * a.group * S * per_row <= kScoreBudget;
  const size_t rows = static_cast<size_t>(a.group) * a.sb * (a.all_groups ? Hkv : 1);
  a.bytes = rup(static_cast<size_t>(Hkv) * Skv * 3 * a.Dp * 4, 256) +        // K'
            rup(static_cast<size_t>(Hkv) * Dh * 3 * a.Kp * 4, 256) +         // V'^T
            rup(rows * 3 * a.Dp * 4, 256) + rup(rows * a.Kp * 4, 256) +     // Q', S
            rup(rows * 3 * a.Kp * 4, 256) +                                   // P'
            (fp8 ? 2 * rup(static_cast<size_t>(Hkv) * Skv * Dh * 4, 256) : 0);
  return a;
}

// Attention on device arrays. K / V: f32 (Kq == nullptr) or e4m3 codes with
// per-head scales.
int attention_device(int S, int Skv, int Dh, int Hq, int Hkv, const float *Q, const float *K,
                     const float *V, const uint8_t *Kq, const uint8_t *Vq, const float *sk,
                     const float *sv, float *O, float scale, int causal, int window, int kv_off,
                     void *ws, size_t ws_bytes, cudaStream_t st) {
  const bool fp8 = Kq != nullptr;
  const AttnPlan a = attn_plan(S, Skv, Dh, Hq, Hkv, fp8);
  if (ws_bytes < a.bytes) return set_status(ROUGE_B200_ETOOBIG);
  Arena ar(ws, ws_bytes);
  const size_t rows = static_cast<size_t>(a.group) * a.sb * (a.all_groups ? Hkv : 1);
  uint32_t *Kp_ = ar.take<uint32_t>(static_cast<size_t>(Hkv) * Skv * 3 * a.Dp);
  uint32_t *Vt = ar.take<uint32_t>(static_cast<size_t>(Hkv) * Dh * 3 * a.Kp);
  uint32_t *Qp = ar.take<uint32_t>(rows * 3 * a.Dp);
  float *Sc = ar.take<float>(rows * a.Kp);
  uint32_t *Pp = ar.take<uint32_t>(rows * 3 * a.Kp);
  int s = ROUGE_B200_OK;
  if (fp8) {
    float *Kd = ar.take<float>(static_cast<size_t>(Hkv) * Skv * Dh);
    float *Vd = ar.take<float>(static_cast<size_t>(Hkv) * Skv * Dh);
    const size_t per = static_cast<size_t>(Skv) * Dh;
    decode_kv_kernel<<<grid_of(per * Hkv), kThreads, 0, st>>>(Kq, per, Hkv, sk, Kd);
    decode_kv_kernel<<<grid_of(per * Hkv), kThreads, 0, st>>>(Vq, per, Hkv, sv, Vd);
    s = cuda_status(cudaGetLastError());
    K = Kd;
    V = Vd;
  }
  // K'[h][t][3Dp] = [hi|lo|hi] of K[h][t][:]; V'^T[h][d][3Kp] = [hi|lo|hi] of V[h][:][d]
  if (s == ROUGE_B200_OK)
    s = pack_launch<uint32_t>(K, static_cast<long long>(Skv) * Dh, Dh, 1, Skv, Dh, a.Dp, 2, Kp_,
                              static_cast<long long>(Skv) * 3 * a.Dp, 3 * a.Dp, Hkv, st);
  if (s == ROUGE_B200_OK)
    s = pack_launch<uint32_t>(V, static_cast<long long>(Skv) * Dh, 1, Dh, Dh, Skv, a.Kp, 2, Vt,
                              static_cast<long long>(Dh) * 3 * a.Kp, 3 * a.Kp, Hkv, st);
  if (a.all_groups) {
    // Every head at once: Q' of all Hq heads ([hk][g][s] rows), the scores
    // of every group as one batched GEMM (item hk: its group's rows times
    // K' of head hk), one softmax pass, and P.V batched the same way; O's
    // [Hq][S][Dh] rows are the same [hk][g][s] order.
    const int m = a.group * S;
    if (s == ROUGE_B200_OK)
      s = pack_launch<uint32_t>(Q, static_cast<long long>(S) * Dh, Dh, 1, S, Dh, a.Dp, 1, Qp,
                                static_cast<long long>(S) * 3 * a.Dp, 3 * a.Dp, Hq, st);
    if (s == ROUGE_B200_OK)
      s = launch_gemm_blas_batched(3, m, Skv, 3 * a.Dp, Qp, 3 * a.Dp, Kp_, 3 * a.Dp, scale, 0.0f,
                                   Sc, a.Kp, Hkv, st);
    if (s == ROUGE_B200_OK) {
      softmax_split_kernel<<<grid_of(static_cast<size_t>(m) * Hkv * 32), kThreads, 0, st>>>(
          Sc, a.Kp, m * Hkv, S, 0, Skv, a.Kp, causal, window, kv_off, Pp);
      s = cuda_status(cudaGetLastError());
    }
    if (s == ROUGE_B200_OK)
      s = launch_gemm_blas_batched(3, m, Dh, 3 * a.Kp, Pp, 3 * a.Kp, Vt, 3 * a.Kp, 1.0f, 0.0f, O,
                                   Dh, Hkv, st);
    return s == ROUGE_B200_OK ? s : set_status(s);
  }
  for (int hk = 0; s == ROUGE_B200_OK && hk < Hkv; ++hk) {
    for (int s0 = 0; s == ROUGE_B200_OK && s0 < S; s0 += a.sb) {
      const int sb = S - s0 < a.sb ? S - s0 : a.sb;
      const int m = a.group * sb;
      // Q'[g * sb + i] = [hi|hi|lo] of Q[hk * group + g][s0 + i]
      s = pack_launch<uint32_t>(Q + (static_cast<size_t>(hk) * a.group * S + s0) * Dh,
                                static_cast<long long>(S) * Dh, Dh, 1, sb, Dh, a.Dp, 1, Qp,
                                static_cast<long long>(sb) * 3 * a.Dp, 3 * a.Dp, a.group, st);
      if (s != ROUGE_B200_OK) break;
      s = launch_gemm_blas(3, m, Skv, 3 * a.Dp, Qp, 3 * a.Dp,
                           Kp_ + static_cast<size_t>(hk) * Skv * 3 * a.Dp, 3 * a.Dp,
                           ROUGE_B200_B_NK, scale, 0.0f, Sc, a.Kp, st);
      if (s != ROUGE_B200_OK) break;
      softmax_split_kernel<<<grid_of(static_cast<size_t>(m) * 32), kThreads, 0, st>>>(
          Sc, a.Kp, m, sb, s0, Skv, a.Kp, causal, window, kv_off, Pp);
      s = cuda_status(cudaGetLastError());
      if (sb == S) {
        // the whole sequence in one block: the group's heads are consecutive
        // [S][Dh] blocks of O, so their P.V products are one GEMM of
        // group * S rows
        s = launch_gemm_blas(3, m, Dh, 3 * a.Kp, Pp, 3 * a.Kp,
                             Vt + static_cast<size_t>(hk) * Dh * 3 * a.Kp, 3 * a.Kp,
                             ROUGE_B200_B_NK, 1.0f, 0.0f,
                             O + static_cast<size_t>(hk) * a.group * S * Dh, Dh, st);
      }
      for (int g = 0; s == ROUGE_B200_OK && sb != S && g < a.group; ++g) {
        const int hq = hk * a.group + g;
        s = launch_gemm_blas(3, sb, Dh, 3 * a.Kp, Pp + static_cast<size_t>(g) * sb * 3 * a.Kp,
                             3 * a.Kp, Vt + static_cast<size_t>(hk) * Dh * 3 * a.Kp, 3 * a.Kp,
                             ROUGE_B200_B_NK, 1.0f, 0.0f,
                             O + (static_cast<size_t>(hq) * S + s0) * Dh, Dh, st);
      }
    }
  }
  return s == ROUGE_B200_OK ? s : set_status(s);
}

// Row-major C[M][N] (pitch ldc) = A[M][K] . W[K][N] + beta * C, f32 through
// the column-major 3xTF32 GEMM (C^T = W^T A^T with no transposes).
int rowmajor_gemm(int M, int N, int K, const float *A, const float *W, float beta, float *C,
                  void *ws, size_t ws_bytes, cudaStream_t st, int lda = 0) {
  return rouge_b200_gemm_colmajor(0, 0, N, M, K, ROUGE_B200_T_F32, 1.0f, W, N, A, lda ? lda : K,
                                  beta, C, ROUGE_B200_T_F32, N, ws, ws_bytes, st);
}

// Workspace of rowmajor_gemm_cat: A' [M][3 Kp] (256-byte aligned), then B'
// [Nt][3 Kp], Kp = K rounded up to the 32-element k-block.
size_t rowmajor_gemm_cat_workspace(int M, int K, int Nt) {
  const size_t Kp = rup(K, 32);
  return rup(static_cast<size_t>(M) * 3 * Kp * 4, 256) + static_cast<size_t>(Nt) * 3 * Kp * 4;
}

// Row-major C[M][sum Nw] = A[M][K] . [W_0 | W_1 | ...] for weights W_j
// [K][Nw_j] (the reference's [in][out]) placed side by side: A packed once,
// each weight packed into its rows of one B' operand, one GEMM.
int rowmajor_gemm_cat(int M, int K, const float *A, int nw, const float *const *W, const int *Nw,
                      float *C, void *ws, size_t ws_bytes, cudaStream_t st) {
  const int Kp = static_cast<int>(rup(K, 32));
  int Nt = 0;
  for (int j = 0; j < nw; ++j) Nt += Nw[j];
  const size_t a_bytes = rup(static_cast<size_t>(M) * 3 * Kp * 4, 256);
  if (ws_bytes < rowmajor_gemm_cat_workspace(M, K, Nt)) return set_status(ROUGE_B200_ETOOBIG);
  uint32_t *Ap = static_cast<uint32_t *>(ws);
  uint32_t *Bp = reinterpret_cast<uint32_t *>(static_cast<uint8_t *>(ws) + a_bytes);
  int s = pack_launch<uint32_t>(A, 0, K, 1, M, K, Kp, 1, Ap, 0, 3 * Kp, 1, st);
  for (int j = 0, off = 0; s == ROUGE_B200_OK && j < nw; off += Nw[j], ++j)
    s = pack_launch<uint32_t>(W[j], 0, 1, Nw[j], Nw[j], K, Kp, 2,
                              Bp + static_cast<size_t>(off) * 3 * Kp, 0, 3 * Kp, 1, st);
  if (s != ROUGE_B200_OK) return s;
  return launch_gemm_blas(3, M, Nt, 3 * Kp, Ap, 3 * Kp, Bp, 3 * Kp, ROUGE_B200_B_NK, 1.0f, 0.0f,
                          C, Nt, st);
}

// GEMM workspace the transformer block needs: the largest of its
// projections' (the q | k | v and gate | up GEMMs through
// rowmajor_gemm_cat, the others through rowmajor_gemm), each sized by the
// function that lays it out.
size_t block_gemm_workspace(int S, int D, int Hq, int Hkv, int Dq, int Dff) {
  size_t g = std::max(rowmajor_gemm_cat_workspace(S, D, (Hq + 2 * Hkv) * Dq),
                      rowmajor_gemm_cat_workspace(S, D, 2 * Dff));
  const int shapes[3][3] = {{Hkv * Dq, S, D}, {D, S, Hq * Dq}, {D, S, Dff}};
  for (auto &sh : shapes)
    g = std::max(g, rouge_b200_gemm_colmajor_workspace(ROUGE_B200_T_F32, sh[0], sh[1], sh[2]));
  return g;
}

}  // namespace
}  // namespace rb200

using namespace rb200;

extern "C" {

size_t rouge_b200_attention_workspace(int S, int Skv, int Dh, int Hq, int Hkv, int fp8_kv) {
  if (S <= 0 || Skv <= 0 || Dh <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv) return 0;
  return attn_plan(S, Skv, Dh, Hq, Hkv, fp8_kv != 0).bytes;
}

int rouge_b200_attention_gqa(int S, int Skv, int Dh, int Hq, int Hkv, const float *Q,
                             const float *K, const float *V, const uint8_t *Kq, const uint8_t *Vq,
                             const float *scales_k, const float *scales_v, float *O, float scale,
                             int causal, int window, int kv_off, void *workspace,
                             size_t workspace_bytes, void *stream) {
  if (!Q || !O || S <= 0 || Skv <= 0 || Dh <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv)
    return set_status(ROUGE_B200_EINVAL);
  const bool fp8 = Kq != nullptr;
  if (fp8 ? (!Vq || !scales_k || !scales_v) : (!K || !V)) return set_status(ROUGE_B200_EINVAL);
  const int s = device_ready();
  if (s != ROUGE_B200_OK) return s;
  if (!(scale > 0.0f)) scale = 1.0f / std::sqrt(static_cast<float>(Dh));  // attention_gqa.cpp:41
  return attention_device(S, Skv, Dh, Hq, Hkv, Q, K, V, Kq, Vq, scales_k, scales_v, O, scale,
                          causal, window, kv_off, workspace, workspace_bytes, as_stream(stream));
}

}  // extern "C"

namespace rb200 {
namespace {

// Host drop-in body of the three attention entries.
void attention_host(int S, int Skv, int Dh, int Hq, int Hkv, const float *Q, const float *K,
                    const float *V, const uint8_t *Kq, const uint8_t *Vq, const float *sk,
                    const float *sv, float *O, float scale, int causal, int window, int kv_off) {
  HostCallContext *ctx = host_context();
  if (!ctx) return;
  std::lock_guard<std::mutex> g(ctx->lock);
  const bool fp8 = Kq != nullptr;
  const size_t nq = static_cast<size_t>(Hq) * S * Dh, nkv = static_cast<size_t>(Hkv) * Skv * Dh;
  const size_t work = attn_plan(S, Skv, Dh, Hq, Hkv, fp8).bytes;
  const size_t need = 2 * rup(nq * 4, 256) + 2 * rup(nkv * (fp8 ? 1 : 4), 256) +
                      (fp8 ? 2 * rup(Hkv * 4, 256) : 0) + work;
  if (ensure_workspace(ctx, need) != ROUGE_B200_OK) return;
  Arena ar(ctx->ws, ctx->ws_bytes);
  float *dQ = ar.take<float>(nq);
  float *dO = ar.take<float>(nq);
  const void *dK = ar.take<uint8_t>(nkv * (fp8 ? 1 : 4));
  const void *dV = ar.take<uint8_t>(nkv * (fp8 ? 1 : 4));
  float *dsk = fp8 ? ar.take<float>(Hkv) : nullptr;
  float *dsv = fp8 ? ar.take<float>(Hkv) : nullptr;
  void *rest = ar.p + ar.used;
  cudaStream_t st = ctx->stream;
  int s = cuda_status(cudaMemcpyAsync(dQ, Q, nq * 4, cudaMemcpyHostToDevice, st));
  if (s == ROUGE_B200_OK)
    s = cuda_status(cudaMemcpyAsync(const_cast<void *>(dK), fp8 ? static_cast<const void *>(Kq) : K,
                                    nkv * (fp8 ? 1 : 4), cudaMemcpyHostToDevice, st));
  if (s == ROUGE_B200_OK)
    s = cuda_status(cudaMemcpyAsync(const_cast<void *>(dV), fp8 ? static_cast<const void *>(Vq) : V,
                                    nkv * (fp8 ? 1 : 4), cudaMemcpyHostToDevice, st));
  if (s == ROUGE_B200_OK && fp8) {
    s = cuda_status(cudaMemcpyAsync(dsk, sk, Hkv * 4, cudaMemcpyHostToDevice, st));
    if (s == ROUGE_B200_OK) s = cuda_status(cudaMemcpyAsync(dsv, sv, Hkv * 4, cudaMemcpyHostToDevice, st));
  }
  if (s == ROUGE_B200_OK)
    s = attention_device(S, Skv, Dh, Hq, Hkv, dQ, fp8 ? nullptr : static_cast<const float *>(dK),
                         fp8 ? nullptr : static_cast<const float *>(dV),
                         fp8 ? static_cast<const uint8_t *>(dK) : nullptr,
                         fp8 ? static_cast<const uint8_t *>(dV) : nullptr, dsk, dsv, dO, scale,
                         causal, window, kv_off, rest, ctx->ws_bytes - ar.used, st);
  if (s == ROUGE_B200_OK) s = cuda_status(cudaMemcpyAsync(O, dO, nq * 4, cudaMemcpyDeviceToHost, st));
  if (s == ROUGE_B200_OK) s = cuda_status(cudaStreamSynchronize(st));
  if (s == ROUGE_B200_OK) take_device_error(st);
}

}  // namespace
}  // namespace rb200

extern "C" {

// attention.cpp:27-88 (one head, no window).
void rouge_attention_f32(int S, int Skv, int D, const float *Q, const float *K, const float *V,
                         float *O, float scale, int causal, int kv_off) {
  if (!Q || !K || !V || !O || S <= 0 || Skv <= 0 || D <= 0) return;
  if (!(scale > 0.0f)) scale = 1.0f / std::sqrt(static_cast<float>(D));
  attention_host(S, Skv, D, 1, 1, Q, K, V, nullptr, nullptr, nullptr, nullptr, O, scale, causal, 0,
                 kv_off);
}

// attention_gqa.cpp:52-163
void rouge_attention_gqa(int S, int Skv, int Dh, int Hq, int Hkv, const float *Q, const float *K,
                         const float *V, float *O, float scale, int causal, int window,
                         int kv_off) {
  if (!Q || !K || !V || !O || S <= 0 || Skv <= 0 || Dh <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv)
    return;
  if (!(scale > 0.0f)) scale = 1.0f / std::sqrt(static_cast<float>(Dh));
  attention_host(S, Skv, Dh, Hq, Hkv, Q, K, V, nullptr, nullptr, nullptr, nullptr, O, scale, causal,
                 window, kv_off);
}

// attention_gqa.cpp:164-269
void rouge_attention_gqa_fp8kv(int S, int Skv, int Dh, int Hq, int Hkv, const float *Q,
                               const uint8_t *Kq, const uint8_t *Vq, const float *scales_k,
                               const float *scales_v, float *O, float scale, int causal,
                               int window, int kv_off) {
  if (!Q || !Kq || !Vq || !scales_k || !scales_v || !O || S <= 0 || Skv <= 0 || Dh <= 0 ||
      Hq <= 0 || Hkv <= 0 || Hq % Hkv)
    return;
  if (!(scale > 0.0f)) scale = 1.0f / std::sqrt(static_cast<float>(Dh));
  attention_host(S, Skv, Dh, Hq, Hkv, Q, nullptr, nullptr, Kq, Vq, scales_k, scales_v, O, scale,
                 causal, window, kv_off);
}

// transformer.cpp:33-68: the single-vector helpers on the device.
void rouge_rmsnorm(const float *x, int n, const float *w, float eps, float *out) {
  if (!x || !w || !out || n <= 0) return;
  HostCallContext *ctx = host_context();
  if (!ctx) return;
  std::lock_guard<std::mutex> g(ctx->lock);
  if (ensure_workspace(ctx, 3 * rup(static_cast<size_t>(n) * 4, 256)) != ROUGE_B200_OK) return;
  Arena ar(ctx->ws, ctx->ws_bytes);
  float *dx = ar.take<float>(n), *dw = ar.take<float>(n), *dout = ar.take<float>(n);
  cudaStream_t st = ctx->stream;
  cudaMemcpyAsync(dx, x, n * 4, cudaMemcpyHostToDevice, st);
  cudaMemcpyAsync(dw, w, n * 4, cudaMemcpyHostToDevice, st);
  rmsnorm_kernel<<<1, 32, 0, st>>>(dx, 1, n, dw, eps, dout);
  if (cuda_status(cudaGetLastError()) == ROUGE_B200_OK)
    cudaMemcpyAsync(out, dout, n * 4, cudaMemcpyDeviceToHost, st);
  cuda_status(cudaStreamSynchronize(st));
}

void rouge_rope(float *x, int heads, int head_dim, int pos, float theta) {
  if (!x || heads <= 0 || head_dim <= 0) return;
  HostCallContext *ctx = host_context();
  if (!ctx) return;
  std::lock_guard<std::mutex> g(ctx->lock);
  const size_t n = static_cast<size_t>(heads) * head_dim;
  if (ensure_workspace(ctx, rup(n * 4, 256)) != ROUGE_B200_OK) return;
  float *dx = static_cast<float *>(ctx->ws);
  cudaStream_t st = ctx->stream;
  cudaMemcpyAsync(dx, x, n * 4, cudaMemcpyHostToDevice, st);
  rope_kernel<<<grid_of(n), kThreads, 0, st>>>(dx, heads, head_dim, pos, theta);
  if (cuda_status(cudaGetLastError()) == ROUGE_B200_OK)
    cudaMemcpyAsync(x, dx, n * 4, cudaMemcpyDeviceToHost, st);
  cuda_status(cudaStreamSynchronize(st));
}

void rouge_swiglu(const float *gate, const float *up, int n, float *out) {
  if (!gate || !up || !out || n <= 0) return;
  HostCallContext *ctx = host_context();
  if (!ctx) return;
  std::lock_guard<std::mutex> g(ctx->lock);
  if (ensure_workspace(ctx, 2 * rup(static_cast<size_t>(n) * 4, 256)) != ROUGE_B200_OK) return;
  Arena ar(ctx->ws, ctx->ws_bytes);
  float *dg = ar.take<float>(n), *du = ar.take<float>(n);
  cudaStream_t st = ctx->stream;
  cudaMemcpyAsync(dg, gate, n * 4, cudaMemcpyHostToDevice, st);
  cudaMemcpyAsync(du, up, n * 4, cudaMemcpyHostToDevice, st);
  swiglu_kernel<<<grid_of(n), kThreads, 0, st>>>(dg, du, n);
  if (cuda_status(cudaGetLastError()) == ROUGE_B200_OK)
    cudaMemcpyAsync(out, dg, n * 4, cudaMemcpyDeviceToHost, st);
  cuda_status(cudaStreamSynchronize(st));
}

// transformer.cpp:79-159 on device arrays (same layouts as the reference).
size_t rouge_b200_transformer_block_workspace(int S, int D, int Hq, int Hkv, int Dq, int Dff) {
  if (S <= 0 || D <= 0 || Hq <= 0 || Hkv <= 0 || Dq <= 0 || Dff <= 0 || Hq % Hkv) return 0;
  const size_t sd = rup(static_cast<size_t>(S) * D * 4, 256);
  const size_t sq = rup(static_cast<size_t>(S) * Hq * Dq * 4, 256);
  const size_t skv = rup(static_cast<size_t>(S) * Hkv * Dq * 4, 256);
  const size_t sf = rup(static_cast<size_t>(S) * Dff * 4, 256);
  const size_t g = block_gemm_workspace(S, D, Hq, Hkv, Dq, Dff);
  return 3 * sd + 4 * sq + 4 * skv + 2 * sf + rup(g, 256) +
         attn_plan(S, S, Dq, Hq, Hkv, false).bytes;
}

int rouge_b200_transformer_block(int S, int D, int Hq, int Hkv, int Dq, int Dk, const float *x,
                                 const float *wrms1, const float *wq, const float *wk,
                                 const float *wv, const float *wo, const float *wrms2,
                                 const float *wgate, const float *wup, const float *wdown, int Dff,
                                 float rope_theta, float rms_eps, float *out, void *workspace,
                                 size_t workspace_bytes, void *stream) {
  if (!x || !out || !wrms1 || !wq || !wk || !wv || !wo || !wrms2 || !wgate || !wup || !wdown ||
      S <= 0 || D <= 0 || Dk != Dq || Dq <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv || Dff <= 0)
    return set_status(ROUGE_B200_EINVAL);
  const size_t need = rouge_b200_transformer_block_workspace(S, D, Hq, Hkv, Dq, Dff);
  if (!workspace || workspace_bytes < need) return set_status(ROUGE_B200_ETOOBIG);
  int s = device_ready();
  if (s != ROUGE_B200_OK) return s;
  cudaStream_t st = as_stream(stream);
  Arena ar(workspace, workspace_bytes);
  const size_t nsd = static_cast<size_t>(S) * D, nq = static_cast<size_t>(S) * Hq * Dq;
  const size_t nkv = static_cast<size_t>(S) * Hkv * Dq, nf = static_cast<size_t>(S) * Dff;
  float *norm = ar.take<float>(nsd), *h1 = ar.take<float>(nsd), *norm2 = ar.take<float>(nsd);
  // qkv [S][(Hq + 2 Hkv) Dq]: the q | k | v projections side by side;
  // gu [S][2 Dff]: gate | up
  float *qkv = ar.take<float>(nq + 2 * nkv), *q = ar.take<float>(nq), *attn = ar.take<float>(nq),
        *attnflat = ar.take<float>(nq);
  float *k = ar.take<float>(nkv), *v = ar.take<float>(nkv);
  float *gu = ar.take<float>(2 * nf);
  const size_t gws = block_gemm_workspace(S, D, Hq, Hkv, Dq, Dff);
  void *gw = ar.take<uint8_t>(gws);
  void *aw = ar.p + ar.used;
  const size_t aw_bytes = workspace_bytes - ar.used;
  const unsigned rows_grid = grid_of(static_cast<size_t>(S) * 32);
  // 1-2: RMSNorm, projections
  rmsnorm_kernel<<<rows_grid, kThreads, 0, st>>>(x, S, D, wrms1, rms_eps, norm);
  s = cuda_status(cudaGetLastError());
  const long long ldqkv = static_cast<long long>(Hq + 2 * Hkv) * Dq;
  if (s == ROUGE_B200_OK) {
    const float *wqkv[3] = {wq, wk, wv};
    const int nqkv[3] = {Hq * Dq, Hkv * Dq, Hkv * Dq};
    s = rowmajor_gemm_cat(S, D, norm, 3, wqkv, nqkv, qkv, gw, gws, st);
  }
  // 3: [S][H*Dq] -> [H][S][Dq], RoPE on q and k (positions 0..S-1)
  if (s == ROUGE_B200_OK) {
    relayout_rope_kernel<<<grid_of(nq), kThreads, 0, st>>>(qkv, ldqkv, S, Hq, Dq, 1, rope_theta, q);
    relayout_rope_kernel<<<grid_of(nkv), kThreads, 0, st>>>(qkv + static_cast<size_t>(Hq) * Dq, ldqkv,
                                                            S, Hkv, Dq, 1, rope_theta, k);
    relayout_rope_kernel<<<grid_of(nkv), kThreads, 0, st>>>(
        qkv + static_cast<size_t>(Hq + Hkv) * Dq, ldqkv, S, Hkv, Dq, 0, rope_theta, v);
    s = cuda_status(cudaGetLastError());
  }
  // 4: causal GQA attention
  if (s == ROUGE_B200_OK)
    s = attention_device(S, S, Dq, Hq, Hkv, q, k, v, nullptr, nullptr, nullptr, nullptr, attn,
                         1.0f / std::sqrt(static_cast<float>(Dq)), 1, 0, 0, aw, aw_bytes, st);
  // 5: h1 = x + attnflat . wo
  if (s == ROUGE_B200_OK) {
    unflatten_kernel<<<grid_of(nq), kThreads, 0, st>>>(attn, S, Hq, Dq, attnflat);
    s = cuda_status(cudaGetLastError());
  }
  if (s == ROUGE_B200_OK) s = cuda_status(cudaMemcpyAsync(h1, x, nsd * 4, cudaMemcpyDeviceToDevice, st));
  if (s == ROUGE_B200_OK) s = rowmajor_gemm(S, D, Hq * Dq, attnflat, wo, 1.0f, h1, gw, gws, st);
  // 6: out = h1 + (silu(norm2 . wgate) * (norm2 . wup)) . wdown
  if (s == ROUGE_B200_OK) {
    rmsnorm_kernel<<<rows_grid, kThreads, 0, st>>>(h1, S, D, wrms2, rms_eps, norm2);
    s = cuda_status(cudaGetLastError());
  }
  if (s == ROUGE_B200_OK) {
    const float *wgu[2] = {wgate, wup};
    const int ngu[2] = {Dff, Dff};
    s = rowmajor_gemm_cat(S, D, norm2, 2, wgu, ngu, gu, gw, gws, st);
  }
  if (s == ROUGE_B200_OK) {
    swiglu_rows_kernel<<<grid_of(nf), kThreads, 0, st>>>(gu, S, Dff);
    s = cuda_status(cudaGetLastError());
  }
  if (s == ROUGE_B200_OK) s = cuda_status(cudaMemcpyAsync(out, h1, nsd * 4, cudaMemcpyDeviceToDevice, st));
  if (s == ROUGE_B200_OK) s = rowmajor_gemm(S, D, Dff, gu, wdown, 1.0f, out, gw, gws, st, 2 * Dff);
  return s == ROUGE_B200_OK ? s : set_status(s);
}

// transformer.cpp:79-159, host pointers (the reference's entry).
void rouge_transformer_block(int S, int D, int Hq, int Hkv, int Dq, int Dk, const float *x,
                             const float *wrms1, const float *wq, const float *wk, const float *wv,
                             const float *wo, const float *wrms2, const float *wgate,
                             const float *wup, const float *wdown, int Dff, float rope_theta,
                             float rms_eps, float *out) {
  if (!x || !out || S <= 0 || D <= 0) return;  // transformer.cpp:85-88
  if (Dk != Dq || Hq <= 0 || Hkv <= 0 || Hq % Hkv != 0 || Dff <= 0) return;
  if (!wrms1 || !wq || !wk || !wv || !wo || !wrms2 || !wgate || !wup || !wdown) return;
  HostCallContext *ctx = host_context();
  if (!ctx) return;
  std::lock_guard<std::mutex> g(ctx->lock);
  const size_t nsd = static_cast<size_t>(S) * D;
  const size_t sizes[11] = {nsd, static_cast<size_t>(D), static_cast<size_t>(D) * Hq * Dq,
                            static_cast<size_t>(D) * Hkv * Dq, static_cast<size_t>(D) * Hkv * Dq,
                            static_cast<size_t>(Hq) * Dq * D, static_cast<size_t>(D),
                            static_cast<size_t>(D) * Dff, static_cast<size_t>(D) * Dff,
                            static_cast<size_t>(Dff) * D, nsd};
  const float *src[10] = {x, wrms1, wq, wk, wv, wo, wrms2, wgate, wup, wdown};
  size_t in_bytes = 0;
  for (size_t n : sizes) in_bytes += rup(n * 4, 256);
  const size_t work = rouge_b200_transformer_block_workspace(S, D, Hq, Hkv, Dq, Dff);
  if (ensure_workspace(ctx, in_bytes + work) != ROUGE_B200_OK) return;
  Arena ar(ctx->ws, ctx->ws_bytes);
  float *d[11];
  for (int i = 0; i < 11; ++i) d[i] = ar.take<float>(sizes[i]);
  cudaStream_t st = ctx->stream;
  int s = ROUGE_B200_OK;
  for (int i = 0; i < 10 && s == ROUGE_B200_OK; ++i)
    s = cuda_status(cudaMemcpyAsync(d[i], src[i], sizes[i] * 4, cudaMemcpyHostToDevice, st));
  if (s == ROUGE_B200_OK)
    s = rouge_b200_transformer_block(S, D, Hq, Hkv, Dq, Dk, d[0], d[1], d[2], d[3], d[4], d[5],
                                     d[6], d[7], d[8], d[9], Dff, rope_theta, rms_eps, d[10],
                                     ar.p + ar.used, ctx->ws_bytes - ar.used, st);
  if (s == ROUGE_B200_OK) s = cuda_status(cudaMemcpyAsync(out, d[10], nsd * 4, cudaMemcpyDeviceToHost, st));
  if (s == ROUGE_B200_OK) s = cuda_status(cudaStreamSynchronize(st));
  if (s == ROUGE_B200_OK) take_device_error(st);
}

}  // extern "C"
