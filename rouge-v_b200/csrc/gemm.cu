// Dense GEMM on sm_100a tensor cores for the rouge-numerics path:
//   kind::i8     int8 x int8 -> exact int32 in TMEM   (rouge_gemm_i8, quant_int8.cpp:189-211)
//   kind::f8f6f4 e4m3 x e4m3 -> f32 in TMEM          (rouge_gemm_e4m3, fp8.cpp:116-124)
//   kind::f16    f16/bf16 -> f32 in TMEM              (rouge_gemm_f16/bf16, fp16.cpp:123-141)
//
// One persistent CTA per SM (grid = min(tiles, SMs)), 256 threads:
//   warp 0      TMA producer: A and B k-blocks into a STAGES-deep ring of
//               128-byte-swizzled shared-memory stages (mbarrier full/empty)
//   warp 1      MMA issuer: one thread issues tcgen05.mma (M=128, N=BN,
//               K=32 bytes per instruction) into a TMEM accumulator and
//               releases each stage with tcgen05.commit
//   warp 2      TMEM allocator (2 x BN columns: double-buffered accumulator)
//   warps 4-7   epilogue: tcgen05.ld of their 32 TMEM lanes, fused scale /
//               dequant / bf16 conversion, predicated global stores; runs
//               while the MMA warp fills the other accumulator
// C tile = 128 x BN. Tiles are walked in groups of 16 M-blocks so that the
// CTAs of one wave share A and B panels in L2.
#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <cstring>

#include "formats.cuh"
#include "x86fp.cuh"
#include "ptx.cuh"
#include "runtime.cuh"

namespace rb200 {
namespace {

constexpr int kBM = 128;
constexpr int kBKBytes = 128;   // one swizzle atom row: 128 B of K per stage row
constexpr int kGroupM = 16;
constexpr int kGemmThreads = 384;  // warps 0-3: producer, MMA, TMEM allocator, idle; 4-11: epilogue

struct GemmArgs {
  int M, N, K;
  int num_m, num_n, num_k, num_tiles;
  void *C;
  long long ldc;
  const float *scales_a;  // int8: per-row or single scale
  const float *scales_b;  // int8: per-column or single scale
  int a_rows, b_cols;
  const float *scale_a;   // e4m3 / f16: per-tensor scale scalars (or null)
  const float *scale_b;
  int bf16;               // kind::f16 inputs are bf16
  int use_tma_store;      // C and ldc are 16-byte aligned: epilogue stores through TMA
  int *err;
  // Implicit-GEMM convolution (A gathered by im2col TMA): M = N*OH*OW
  // output pixels, K = KH*KW*Cin ordered (kr, kc, c), k-block = one filter
  // tap x 64 channels.
  const float *bias;      // per output channel (column) bias added in the epilogue, or null
  int conv_cblocks;       // Cin / 64
  int conv_kw, conv_oh, conv_ow, conv_stride, conv_pad, conv_cin;
};

constexpr int kStageBytes = 4096;  // one epilogue staging buffer (32 rows x 128 B)

template <MmaKind KIND, int BN, bool B_MN>
struct Cfg {
  static constexpr int ESIZE = KIND == MmaKind::F16 ? 2 : 1;
  static constexpr int BK = kBKBytes / ESIZE;       // elements of K per stage
  static constexpr int UMMA_K = 32 / ESIZE;         // elements of K per instruction
  static constexpr int A_BYTES = kBM * kBKBytes;
  static constexpr int B_BYTES = BN * kBKBytes;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (192 * 1024) / STAGE_BYTES > 8 ? 8 : (192 * 1024) / STAGE_BYTES;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int B_CHUNKS = (BN * ESIZE) / kBKBytes;  // 128-byte N chunks (MN-major B)
  static constexpr int B_CHUNK_BYTES = B_MN ? BK * kBKBytes : B_BYTES;
  static constexpr int BAR_BYTES = 256;
  static constexpr int EPI_BYTES = 8 * kStageBytes;  // one staging buffer per epilogue warp
  static constexpr int SMEM = 1024 + STAGES * STAGE_BYTES + EPI_BYTES + BAR_BYTES;
  static_assert(SMEM <= 232448, "exceeds the 227 KB per-CTA shared memory limit");
  static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "BN");
  static_assert(TMEM_COLS == 64 || TMEM_COLS == 128 || TMEM_COLS == 256 || TMEM_COLS == 512,
                "TMEM allocation must be a power of two >= 32");
};

__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int &mb, int &nb) {
  const int group = t / (kGroupM * num_n);
  const int first_m = group * kGroupM;
  const int rows_in_group = min(num_m - first_m, kGroupM);
  const int r = t - group * kGroupM * num_n;
  mb = first_m + r % rows_in_group;
  nb = r / rows_in_group;
}

__device__ __forceinline__ void report(int *err, volatile int *abort, int code) {
  *abort = 1;
  if (err) atomicCAS(err, 0, code);
}

// Converts one 32-column chunk of one warp's 32 accumulator rows (thread =
// row, v[j] = column col0 + j) and writes it to C.
//   TMA path: the chunk goes to a 128-byte (f32/i32) or 64-byte (bf16)
//   swizzled staging buffer in shared memory and one lane issues a tiled
//   TMA store of the 32 x 32 box; out-of-range rows and columns are
//   clipped by the tensor map. Two buffers alternate per warp.
//   Direct path (C not 16-byte aligned): predicated per-thread stores.
template <MmaKind KIND, int OUT>
__device__ __forceinline__ void epilogue_chunk(const GemmArgs &args, const uint32_t (&v)[32],
                                               int col0, int row0, int row, bool row_ok, float sa,
                                               bool sa_ok, float sab, uint8_t *buf,
                                               const CUtensorMap *tmC, int lane) {
  uint32_t o[32];  // f32 / i32 bits, or bf16 pairs in o[0..15]
  if constexpr (OUT == ROUGE_B200_OUT_I32) {
#pragma unroll
    for (int j = 0; j < 32; ++j) o[j] = v[j];
  } else {
    float f[32];
    bool may_nan = true;
    if constexpr (KIND == MmaKind::I8) {
      float sbl;  // scale of column col0 + lane
      if (args.b_cols) {
        const int col = col0 + lane;
        sbl = col < args.N ? __ldg(args.scales_b + col) : 0.0f;
      } else {
        sbl = __ldg(args.scales_b);
      }
      // With sa and every column scale of the chunk finite and below 2^96,
      // (float)acc * sa is finite (|acc| < 2^31) and the second product can
      // only overflow to +-inf, which x86 and the GPU both produce: no NaN,
      // so the plain multiplies are exact here.
      const bool fast = __all_sync(0xffffffffu, sa_ok && fabsf(sbl) < 7.9e28f);
      may_nan = !fast;
      // quant_int8.cpp:208: ((float)acc * sa) * sb, two rounded multiplies
      if (fast) {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float sb = args.b_cols ? __shfl_sync(0xffffffffu, sbl, j) : sbl;
          f[j] = __fmul_rn(__fmul_rn(__int2float_rn(static_cast<int32_t>(v[j])), sa), sb);
        }
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float sb = args.b_cols ? __shfl_sync(0xffffffffu, sbl, j) : sbl;
          f[j] = x86_mul(x86_mul(__int2float_rn(static_cast<int32_t>(v[j])), sa), sb);
        }
      }
    } else if (args.bias) {
      // conv.cpp:61-64: bias added to the finished f32 sum of each channel
      const int col = col0 + lane;
      const float bl = col < args.N ? __ldg(args.bias + col) : 0.0f;
#pragma unroll
      for (int j = 0; j < 32; ++j)
        f[j] = __fadd_rn(__uint_as_float(v[j]), __shfl_sync(0xffffffffu, bl, j));
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) f[j] = __fmul_rn(__uint_as_float(v[j]), sab);
    }
    if constexpr (OUT == ROUGE_B200_OUT_F32) {
#pragma unroll
      for (int j = 0; j < 32; ++j) o[j] = __float_as_uint(f[j]);
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) o[j] = bf16x2_rn(f[2 * j], f[2 * j + 1]);
      if (may_nan) {  // the reference writes every NaN as 0x7fc0 (fp16.cpp:106)
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          if (isnan(f[2 * j])) o[j] = (o[j] & 0xFFFF0000u) | 0x7FC0u;
          if (isnan(f[2 * j + 1])) o[j] = (o[j] & 0x0000FFFFu) | 0x7FC00000u;
        }
      }
    }
  }

  if (args.use_tma_store) {
    if (lane == 0) bulk_wait_read<0>();  // this warp's previous store has read the buffer
    __syncwarp();
    const uint32_t base = smem_u32(buf);
    if constexpr (OUT == ROUGE_B200_OUT_BF16) {
      const uint32_t r = base + static_cast<uint32_t>(lane) * 64u;  // 64-byte swizzle atoms
      const uint32_t x = (static_cast<uint32_t>(lane) >> 1) & 3u;
#pragma unroll
      for (int k = 0; k < 4; ++k)
        st_shared_v4(r + ((static_cast<uint32_t>(k) ^ x) << 4), o[4 * k], o[4 * k + 1],
                     o[4 * k + 2], o[4 * k + 3]);
    } else {
      const uint32_t r = base + static_cast<uint32_t>(lane) * 128u;  // 128-byte swizzle atoms
      const uint32_t x = static_cast<uint32_t>(lane) & 7u;
#pragma unroll
      for (int k = 0; k < 8; ++k)
        st_shared_v4(r + ((static_cast<uint32_t>(k) ^ x) << 4), o[4 * k], o[4 * k + 1],
                     o[4 * k + 2], o[4 * k + 3]);
    }
    fence_async_smem();
    __syncwarp();
    if (lane == 0) {
      if (row0 < args.M) tma_store_2d(tmC, buf, col0, row0);
      bulk_commit();
    }
    return;
  }

  if (!row_ok) return;
  const bool full_chunk = col0 + 32 <= args.N;
  if constexpr (OUT == ROUGE_B200_OUT_BF16) {
    uint16_t *crow = static_cast<uint16_t *>(args.C) + static_cast<long long>(row) * args.ldc + col0;
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (full_chunk || col0 + j < args.N)
        crow[j] = static_cast<uint16_t>(o[j >> 1] >> ((j & 1) * 16));
  } else {
    uint32_t *crow = static_cast<uint32_t *>(args.C) + static_cast<long long>(row) * args.ldc + col0;
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (full_chunk || col0 + j < args.N) crow[j] = o[j];
  }
}

template <MmaKind KIND, int BN, bool B_MN, int OUT, bool CONV = false>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmC, const GemmArgs args) {
  using C = Cfg<KIND, BN, B_MN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~static_cast<uintptr_t>(1023));
  uint8_t *sA = smem;
  uint8_t *sB = smem + C::STAGES * C::A_BYTES;
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + C::STAGES * C::STAGE_BYTES + C::EPI_BYTES);
  uint64_t *empty = full + C::STAGES;
  uint64_t *tfull = empty + C::STAGES;  // [2]
  uint64_t *tempty = tfull + 2;         // [2]
  uint64_t *mdone = tempty + 2;         // [1] drain barrier for the abort path
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(mdone + 1);
  volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 8);  // one arrival per epilogue warp
    }
    mbar_init(mdone, 1);
    *abort = 0;
    mbar_init_fence();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ producer
    int it = 0;
    bool ok = true;
    for (int t = blockIdx.x; ok && t < args.num_tiles; t += gridDim.x) {
      int mb, nb;
      tile_coords(t, args.num_m, args.num_n, mb, nb);
      // Convolution: box position of the tile's first output pixel.
      int cw = 0, ch = 0, cn = 0;
      if constexpr (CONV) {
        const int p0 = mb * kBM, ohw = args.conv_oh * args.conv_ow;
        cn = p0 / ohw;
        const int rem = p0 - cn * ohw;
        ch = (rem / args.conv_ow) * args.conv_stride - args.conv_pad;
        cw = (rem % args.conv_ow) * args.conv_stride - args.conv_pad;
      }
      for (int kb = 0; kb < args.num_k; ++kb, ++it) {
        const int s = it % C::STAGES;
        const uint32_t round = static_cast<uint32_t>(it / C::STAGES);
        if (!mbar_wait(&empty[s], (round & 1u) ^ 1u, abort)) {
          report(args.err, abort, ROUGE_B200_ETIMEOUT);
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&full[s], C::STAGE_BYTES);
        int kx = kb * C::BK;  // K coordinate of the B tile
        if constexpr (CONV) {
          const int tap = kb / args.conv_cblocks;
          const int c0 = (kb - tap * args.conv_cblocks) * C::BK;
          const int kr = tap / args.conv_kw, kc = tap - kr * args.conv_kw;
          tma_load_im2col_4d(sA + s * C::A_BYTES, &tmA, &full[s], c0, cw, ch, cn,
                             static_cast<uint16_t>(kc), static_cast<uint16_t>(kr));
          kx = tap * args.conv_cin + c0;
        } else {
          tma_load_2d(sA + s * C::A_BYTES, &tmA, &full[s], kx, mb * kBM);
        }
        if constexpr (!B_MN) {
          tma_load_2d(sB + s * C::B_BYTES, &tmB, &full[s], kx, nb * BN);
        } else {
#pragma unroll
          for (int j = 0; j < C::B_CHUNKS; ++j)
            tma_load_2d(sB + s * C::B_BYTES + j * C::B_CHUNK_BYTES, &tmB, &full[s],
                        nb * BN + j * (kBKBytes / C::ESIZE), kb * C::BK);
        }
      }
    }
    if (!ok) {
      // Let the loads already issued land before the CTA's shared memory is
      // released: the last STAGES iterations are the only ones in flight.
      for (int j = (it > C::STAGES ? it - C::STAGES : 0); j < it; ++j) {
        const volatile int never = 0;
        mbar_wait(&full[j % C::STAGES], static_cast<uint32_t>(j / C::STAGES) & 1u, &never);
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------------------ MMA issuer
    constexpr uint32_t c_fmt = KIND == MmaKind::I8 ? 2u : 1u;  // S32 : F32
    constexpr uint32_t ab_fmt = KIND == MmaKind::I8 ? 1u : 0u;  // S8 / E4M3 / F16
    const uint32_t ab = (KIND == MmaKind::F16 && args.bf16) ? 1u : ab_fmt;
    const uint32_t idesc = make_idesc(c_fmt, ab, ab, 0u, B_MN ? 1u : 0u, kBM, BN);
    int it = 0, local = 0;
    bool ok = true;
    bool issued = false;
    for (int t = blockIdx.x; ok && t < args.num_tiles; t += gridDim.x, ++local) {
      const int slot = local & 1;
      const uint32_t use = static_cast<uint32_t>(local >> 1);
      if (!mbar_wait(&tempty[slot], (use & 1u) ^ 1u, abort)) {
        report(args.err, abort, ROUGE_B200_ETIMEOUT);
        ok = false;
        break;
      }
      tc_fence_after_sync();
      const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(slot * BN);
      for (int kb = 0; kb < args.num_k; ++kb, ++it) {
        const int s = it % C::STAGES;
        const uint32_t round = static_cast<uint32_t>(it / C::STAGES);
        if (!mbar_wait(&full[s], round & 1u, abort)) {
          report(args.err, abort, ROUGE_B200_ETIMEOUT);
          ok = false;
          break;
        }
        tc_fence_after_sync();
        const uint32_t a0 = smem_u32(sA + s * C::A_BYTES);
        const uint32_t b0 = smem_u32(sB + s * C::B_BYTES);
#pragma unroll
        for (int k = 0; k < C::BK / C::UMMA_K; ++k) {
          const uint64_t adesc = smem_desc_sw128(a0 + k * 32, 16, 1024);
          const uint64_t bdesc =
              B_MN ? smem_desc_sw128(b0 + k * C::UMMA_K * kBKBytes, C::B_CHUNK_BYTES, 1024)
                   : smem_desc_sw128(b0 + k * 32, 16, 1024);
          umma<KIND>(d_tmem, adesc, bdesc, idesc, (kb | k) != 0 ? 1u : 0u);
        }
        issued = true;
        tc_commit(&empty[s]);
      }
      if (!ok) break;
      tc_commit(&tfull[slot]);
    }
    if (!ok && issued) {
      // Drain the MMAs already issued before TMEM is released.
      const volatile int never = 0;
      tc_commit(mdone);
      mbar_wait(mdone, 0u, &never);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ epilogue
    // Eight warps: warp w reads TMEM lanes [32*(w%4), +32) (the lane quarter
    // its position in the warpgroup allows) and half h = (w-4)/4 of the
    // tile's columns. One 4 KB staging buffer per warp for its TMA stores.
    const int quarter = warp & 3;
    const int half = (warp - 4) >> 2;
    uint8_t *stage = smem + C::STAGES * C::STAGE_BYTES + (warp - 4) * kStageBytes;
    int local = 0;
    float sab = 1.0f;
    if constexpr (KIND != MmaKind::I8) {
      if (args.scale_a && args.scale_b) sab = x86_mul(__ldg(args.scale_a), __ldg(args.scale_b));
    }
    for (int t = blockIdx.x; t < args.num_tiles; t += gridDim.x, ++local) {
      int mb, nb;
      tile_coords(t, args.num_m, args.num_n, mb, nb);
      const int slot = local & 1;
      const uint32_t use = static_cast<uint32_t>(local >> 1);
      if (!mbar_wait(&tfull[slot], use & 1u, abort)) {
        report(args.err, abort, ROUGE_B200_ETIMEOUT);
        break;
      }
      tc_fence_after_sync();
      const int row0 = mb * kBM + quarter * 32;
      const int row = row0 + lane;
      const bool row_ok = row < args.M;
      float sa = 1.0f;
      if constexpr (KIND == MmaKind::I8) {
        if (OUT != ROUGE_B200_OUT_I32 && row_ok) sa = __ldg(args.scales_a + (args.a_rows ? row : 0));
      }
      const bool sa_ok = fabsf(sa) < 7.9e28f;  // finite and below 2^96
      const uint32_t tbase =
          tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(slot * BN);
      const int cols_left = args.N - nb * BN;
      const int nchunks = cols_left >= BN ? BN / 32 : (cols_left + 31) / 32;  // warp-uniform
      const int c_end = min(nchunks, (half + 1) * (BN / 64));
      const int c_beg = half * (BN / 64);
      if (c_beg < c_end) {
        uint32_t va[32], vb[32];
        tmem_ld_32x32b_x32(tbase + static_cast<uint32_t>(c_beg * 32), va);
        tmem_ld_wait_regs(va);
        for (int c = c_beg; c < c_end; c += 2) {
          // The load of chunk c+1 is in flight while chunk c is converted and stored.
          if (c + 1 < c_end) tmem_ld_32x32b_x32(tbase + static_cast<uint32_t>((c + 1) * 32), vb);
          epilogue_chunk<KIND, OUT>(args, va, nb * BN + c * 32, row0, row, row_ok, sa, sa_ok, sab,
                                    stage, &tmC, lane);
          if (c + 1 < c_end) {
            tmem_ld_wait_regs(vb);
            if (c + 2 < c_end) tmem_ld_32x32b_x32(tbase + static_cast<uint32_t>((c + 2) * 32), va);
            epilogue_chunk<KIND, OUT>(args, vb, nb * BN + (c + 1) * 32, row0, row, row_ok, sa,
                                      sa_ok, sab, stage, &tmC, lane);
            if (c + 2 < c_end) tmem_ld_wait_regs(va);
          }
        }
      }
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[slot]);
    }
    if (args.use_tma_store && lane == 0) bulk_wait_all();
  }

  tc_fence_before_sync();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after_sync();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// Builds the output map and launches one GEMM / convolution.
template <MmaKind KIND, int BN, bool B_MN, int OUT, bool CONV>
int launch_tiles(const CUtensorMap &ta, const CUtensorMap &tb, GemmArgs args, cudaStream_t st) {
  using C = Cfg<KIND, BN, B_MN>;
  int s = ROUGE_B200_OK;
  // Output map for the epilogue's TMA stores: 32 x 32 boxes, swizzle
  // matching the staging layout (128 B rows for 4-byte, 64 B for bf16).
  CUtensorMap tc;
  std::memset(&tc, 0, sizeof(tc));
  if (args.use_tma_store) {
    const bool b16 = OUT == ROUGE_B200_OUT_BF16;
    s = make_tmap_2d(&tc, args.C,
                     b16 ? CU_TENSOR_MAP_DATA_TYPE_UINT16 : CU_TENSOR_MAP_DATA_TYPE_UINT32, args.N,
                     args.M, static_cast<uint64_t>(args.ldc) * (b16 ? 2 : 4), 32, 32,
                     b16 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B);
    if (s != ROUGE_B200_OK) return s;
  }

  auto kern = gemm_tc_kernel<KIND, BN, B_MN, OUT, CONV>;
  // The shared-memory opt-in is a per-device function attribute.
  static std::atomic<unsigned long long> attr_done{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const unsigned long long bit = 1ull << (dev & 63);
  if (!(attr_done.load() & bit)) {
    s = cuda_status(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
    if (s != ROUGE_B200_OK) return s;
    attr_done.fetch_or(bit);
  }
  const int sms = current_sm_count();
  const int grid = args.num_tiles < sms ? args.num_tiles : sms;
  kern<<<grid, kGemmThreads, C::SMEM, st>>>(ta, tb, tc, args);
  return cuda_status(cudaGetLastError());
}

template <MmaKind KIND, int BN, bool B_MN, int OUT>
int launch_gemm_impl(const void *A, long long lda, const void *B, long long ldb, GemmArgs args,
                     cudaStream_t st) {
  using C = Cfg<KIND, BN, B_MN>;
  const CUtensorMapDataType dt =
      C::ESIZE == 2 ? CU_TENSOR_MAP_DATA_TYPE_UINT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8;
  CUtensorMap ta, tb;
  int s = make_tmap_2d(&ta, A, dt, args.K, args.M, static_cast<uint64_t>(lda) * C::ESIZE, C::BK,
                       kBM);
  if (s != ROUGE_B200_OK) return s;
  if (!B_MN)
    s = make_tmap_2d(&tb, B, dt, args.K, args.N, static_cast<uint64_t>(ldb) * C::ESIZE, C::BK, BN);
  else
    s = make_tmap_2d(&tb, B, dt, args.N, args.K, static_cast<uint64_t>(ldb) * C::ESIZE,
                     kBKBytes / C::ESIZE, C::BK);
  if (s != ROUGE_B200_OK) return s;
  return launch_tiles<KIND, BN, B_MN, OUT, false>(ta, tb, args, st);
}

template <MmaKind KIND, int BN, bool B_MN>
int launch_out(const void *A, long long lda, const void *B, long long ldb, GemmArgs args,
               int out_type, cudaStream_t st) {
  switch (out_type) {
    case ROUGE_B200_OUT_F32:
      return launch_gemm_impl<KIND, BN, B_MN, ROUGE_B200_OUT_F32>(A, lda, B, ldb, args, st);
    case ROUGE_B200_OUT_BF16:
      return launch_gemm_impl<KIND, BN, B_MN, ROUGE_B200_OUT_BF16>(A, lda, B, ldb, args, st);
    default:
      if constexpr (KIND == MmaKind::I8)
        return launch_gemm_impl<KIND, BN, B_MN, ROUGE_B200_OUT_I32>(A, lda, B, ldb, args, st);
      return set_status(ROUGE_B200_EINVAL);
  }
}

template <MmaKind KIND>
int launch_kind(const void *A, long long lda, const void *B, long long ldb, int b_layout,
                GemmArgs args, int out_type, cudaStream_t st) {
  // BN = 256 unless that leaves most SMs idle; then 128.
  const int sms = current_sm_count();
  const long long tiles256 =
      static_cast<long long>((args.M + kBM - 1) / kBM) * ((args.N + 255) / 256);
#ifdef RB200_FORCE_BN  // compile-time tile override for tuning builds
  const int bn = RB200_FORCE_BN;
  (void)tiles256;
  (void)sms;
#else
  const int bn = tiles256 >= sms ? 256 : 128;
#endif
  args.num_m = (args.M + kBM - 1) / kBM;
  args.num_n = (args.N + bn - 1) / bn;
  const int esize = KIND == MmaKind::F16 ? 2 : 1;
  const int bk = kBKBytes / esize;
  args.num_k = (args.K + bk - 1) / bk;
  args.num_tiles = args.num_m * args.num_n;
  const bool mn = b_layout == ROUGE_B200_B_KN;
  if (bn == 256)
    return mn ? launch_out<KIND, 256, true>(A, lda, B, ldb, args, out_type, st)
              : launch_out<KIND, 256, false>(A, lda, B, ldb, args, out_type, st);
  return mn ? launch_out<KIND, 128, true>(A, lda, B, ldb, args, out_type, st)
            : launch_out<KIND, 128, false>(A, lda, B, ldb, args, out_type, st);
}

int check_common(int M, int N, int K, const void *A, const void *B, const void *Cp, int ldc,
                 int b_layout, int out_type, int esize) {
  if (M <= 0 || N <= 0 || K <= 0 || !A || !B || !Cp || ldc < N) return ROUGE_B200_EINVAL;
  if (b_layout != ROUGE_B200_B_KN && b_layout != ROUGE_B200_B_NK) return ROUGE_B200_EINVAL;
  if (out_type != ROUGE_B200_OUT_F32 && out_type != ROUGE_B200_OUT_BF16 &&
      out_type != ROUGE_B200_OUT_I32)
    return ROUGE_B200_EINVAL;
  // TMA: 16-byte aligned bases and row pitches.
  if ((reinterpret_cast<uintptr_t>(A) & 15u) || (reinterpret_cast<uintptr_t>(B) & 15u))
    return ROUGE_B200_EUNSUPPORTED;
  if ((static_cast<long long>(K) * esize) % 16) return ROUGE_B200_EUNSUPPORTED;
  if (b_layout == ROUGE_B200_B_KN && (static_cast<long long>(N) * esize) % 16)
    return ROUGE_B200_EUNSUPPORTED;
  return ROUGE_B200_OK;
}

int vec_ok(const void *Cp, long long ldc, int out_type) {
  const int es = out_type == ROUGE_B200_OUT_BF16 ? 2 : 4;
  return ((reinterpret_cast<uintptr_t>(Cp) & 15u) == 0 && (static_cast<long long>(ldc) * es) % 16 == 0)
             ? 1
             : 0;
}

template <int BN>
int launch_conv_bn(const CUtensorMap &ta, const uint16_t *Wt, GemmArgs g, cudaStream_t st) {
  CUtensorMap tb;
  int s = make_tmap_2d(&tb, Wt, CU_TENSOR_MAP_DATA_TYPE_UINT16, g.K, g.N,
                       static_cast<uint64_t>(g.K) * 2, 64, BN);
  if (s != ROUGE_B200_OK) return s;
  return launch_tiles<MmaKind::F16, BN, false, ROUGE_B200_OUT_F32, true>(ta, tb, g, st);
}

}  // namespace

// Implicit-GEMM convolution, NHWC f16/bf16 in, f32 NHWC out (+ bias).
// GEMM view: M = N*OH*OW output pixels, N = Cout, K = KH*KW*Cin in
// (kr, kc, c) order, so the weights [Cout][KH][KW][Cin] are the K-major B
// operand as stored. The A tile of k-block (tap, c0) is one im2col TMA load:
// 128 consecutive output pixels (crossing rows and images) x 64 channels of
// filter tap (kr, kc), zeros in the padding.
int launch_conv_f16(int N, int H, int W, int Cin, int Cout, int KH, int KW, int stride, int pad,
                    const uint16_t *X, const uint16_t *Wt, const float *bias, float *Y,
                    int is_bf16, cudaStream_t st) {
  const int OH = (H + 2 * pad - KH) / stride + 1, OW = (W + 2 * pad - KW) / stride + 1;
  GemmArgs g{};
  g.M = N * OH * OW;
  g.N = Cout;
  g.K = KH * KW * Cin;
  g.C = Y;
  g.ldc = Cout;
  g.bf16 = is_bf16 ? 1 : 0;
  g.bias = bias;
  g.use_tma_store = vec_ok(Y, Cout, ROUGE_B200_OUT_F32);
  g.err = device_error_word();
  g.conv_cblocks = Cin / 64;
  g.conv_kw = KW;
  g.conv_oh = OH;
  g.conv_ow = OW;
  g.conv_stride = stride;
  g.conv_pad = pad;
  g.conv_cin = Cin;
  CUtensorMap ta;
  int s = make_tmap_im2col_nhwc(&ta, X, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, N, H, W, Cin, -pad, -pad,
                                pad - (KW - 1), pad - (KH - 1), 64, kBM, stride, stride);
  if (s != ROUGE_B200_OK) return s;
  const int sms = current_sm_count();
  const long long tiles256 = static_cast<long long>((g.M + kBM - 1) / kBM) * ((Cout + 255) / 256);
  const int bn = (Cout > 128 && tiles256 >= sms) ? 256 : 128;
  g.num_m = (g.M + kBM - 1) / kBM;
  g.num_n = (Cout + bn - 1) / bn;
  g.num_k = KH * KW * g.conv_cblocks;
  g.num_tiles = g.num_m * g.num_n;
  return bn == 256 ? launch_conv_bn<256>(ta, Wt, g, st) : launch_conv_bn<128>(ta, Wt, g, st);
}

int launch_gemm_i8(int M, int N, int K, const int8_t *A, long long lda, const int8_t *B,
                   long long ldb, int b_layout, const float *sa, int a_rows, const float *sb,
                   int b_cols, void *Cp, long long ldc, int out_type, cudaStream_t st) {
  GemmArgs g{};
  g.M = M; g.N = N; g.K = K;
  g.C = Cp; g.ldc = ldc;
  g.scales_a = sa; g.scales_b = sb; g.a_rows = a_rows; g.b_cols = b_cols;
  g.use_tma_store = vec_ok(Cp, ldc, out_type);
  g.err = device_error_word();
  return launch_kind<MmaKind::I8>(A, lda, B, ldb, b_layout, g, out_type, st);
}

// As launch_gemm_i8, with the device word that receives a timeout status
// supplied by the caller.
int launch_gemm_i8_with_err(int M, int N, int K, const int8_t *A, long long lda, const int8_t *B,
                            long long ldb, int b_layout, const float *sa, int a_rows,
                            const float *sb, int b_cols, void *Cp, long long ldc, int out_type,
                            int *err, cudaStream_t st) {
  GemmArgs g{};
  g.M = M; g.N = N; g.K = K;
  g.C = Cp; g.ldc = ldc;
  g.scales_a = sa; g.scales_b = sb; g.a_rows = a_rows; g.b_cols = b_cols;
  g.use_tma_store = vec_ok(Cp, ldc, out_type);
  g.err = err;
  return launch_kind<MmaKind::I8>(A, lda, B, ldb, b_layout, g, out_type, st);
}

int launch_gemm_e4m3(int M, int N, int K, const uint8_t *A, long long lda, const uint8_t *B,
                     long long ldb, int b_layout, const float *scale_a, const float *scale_b,
                     void *Cp, long long ldc, int out_type, cudaStream_t st) {
  GemmArgs g{};
  g.M = M; g.N = N; g.K = K;
  g.C = Cp; g.ldc = ldc;
  g.scale_a = scale_a; g.scale_b = scale_b;
  g.use_tma_store = vec_ok(Cp, ldc, out_type);
  g.err = device_error_word();
  return launch_kind<MmaKind::F8F6F4>(A, lda, B, ldb, b_layout, g, out_type, st);
}

int launch_gemm_f16(int M, int N, int K, const uint16_t *A, long long lda, const uint16_t *B,
                    long long ldb, int b_layout, int is_bf16, void *Cp, long long ldc,
                    int out_type, cudaStream_t st) {
  GemmArgs g{};
  g.M = M; g.N = N; g.K = K;
  g.C = Cp; g.ldc = ldc;
  g.bf16 = is_bf16 ? 1 : 0;
  g.use_tma_store = vec_ok(Cp, ldc, out_type);
  g.err = device_error_word();
  return launch_kind<MmaKind::F16>(A, lda, B, ldb, b_layout, g, out_type, st);
}

}  // namespace rb200

using namespace rb200;

extern "C" {

int rouge_b200_gemm_i8(int M, int N, int K, const int8_t *A, const int8_t *B, int b_layout,
                       const float *scales_a, int a_rows, const float *scales_b, int b_cols,
                       void *C, int ldc, int out_type, void *stream) {
  int s = check_common(M, N, K, A, B, C, ldc, b_layout, out_type, 1);
  if (s != ROUGE_B200_OK) return set_status(s);
  if (out_type != ROUGE_B200_OUT_I32 && (!scales_a || !scales_b)) return set_status(ROUGE_B200_EINVAL);
  s = device_ready();
  if (s != ROUGE_B200_OK) return s;
  const long long ldb = b_layout == ROUGE_B200_B_KN ? N : K;
  return launch_gemm_i8(M, N, K, A, K, B, ldb, b_layout, scales_a, a_rows, scales_b, b_cols, C,
                        ldc, out_type, as_stream(stream));
}

int rouge_b200_gemm_e4m3(int M, int N, int K, const uint8_t *A, const uint8_t *B, int b_layout,
                         const float *scale_a, const float *scale_b, void *C, int ldc,
                         int out_type, void *stream) {
  int s = check_common(M, N, K, A, B, C, ldc, b_layout, out_type, 1);
  if (s != ROUGE_B200_OK) return set_status(s);
  if (out_type == ROUGE_B200_OUT_I32 || (!scale_a) != (!scale_b)) return set_status(ROUGE_B200_EINVAL);
  s = device_ready();
  if (s != ROUGE_B200_OK) return s;
  const long long ldb = b_layout == ROUGE_B200_B_KN ? N : K;
  return launch_gemm_e4m3(M, N, K, A, K, B, ldb, b_layout, scale_a, scale_b, C, ldc, out_type,
                          as_stream(stream));
}

int rouge_b200_conv2d_nhwc_f16(int N, int H, int W, int Cin, int Cout, int KH, int KW, int stride,
                               int pad, const uint16_t *X, const uint16_t *Wt, const float *bias,
                               float *Y, int is_bf16, void *stream) {
  if (!X || !Wt || !Y || N <= 0 || H <= 0 || W <= 0 || Cin <= 0 || Cout <= 0 || KH <= 0 ||
      KW <= 0 || stride <= 0 || pad < 0)
    return set_status(ROUGE_B200_EINVAL);
  const long long OH = (static_cast<long long>(H) + 2 * pad - KH) / stride + 1;
  const long long OW = (static_cast<long long>(W) + 2 * pad - KW) / stride + 1;
  if (OH <= 0 || OW <= 0) return set_status(ROUGE_B200_EINVAL);  // conv.cpp:249
  // im2col TMA limits: 64-channel boxes, corners in [-128, 127], filter
  // offsets below 256, traversal stride up to 8; inputs of at least 128 KB.
  const long long xbytes = static_cast<long long>(N) * H * W * Cin * 2;
  if (Cin % 64 || Cout % 4 || pad > 128 || pad - (KW - 1) < -128 || pad - (KH - 1) < -128 ||
      KH > 256 || KW > 256 || stride > 8 || xbytes < 131072 ||
      static_cast<long long>(N) * OH * OW > 0x7fffffffLL ||
      (reinterpret_cast<uintptr_t>(X) & 15u) || (reinterpret_cast<uintptr_t>(Wt) & 15u))
    return set_status(ROUGE_B200_EUNSUPPORTED);
  int s = device_ready();
  if (s != ROUGE_B200_OK) return s;
  return launch_conv_f16(N, H, W, Cin, Cout, KH, KW, stride, pad, X, Wt, bias, Y, is_bf16,
                         as_stream(stream));
}

int rouge_b200_gemm_f16(int M, int N, int K, const uint16_t *A, const uint16_t *B, int b_layout,
                        int is_bf16, void *C, int ldc, int out_type, void *stream) {
  int s = check_common(M, N, K, A, B, C, ldc, b_layout, out_type, 2);
  if (s != ROUGE_B200_OK) return set_status(s);
  if (out_type == ROUGE_B200_OUT_I32) return set_status(ROUGE_B200_EINVAL);
  s = device_ready();
  if (s != ROUGE_B200_OK) return s;
  const long long ldb = b_layout == ROUGE_B200_B_KN ? N : K;
  return launch_gemm_f16(M, N, K, A, K, B, ldb, b_layout, is_bf16, C, ldc, out_type,
                         as_stream(stream));
}

}  // extern "C"
