// Dense GEMM on sm_100a tensor cores for the rouge-numerics path:
//   kind::i8     int8 x int8 -> exact int32 in TMEM   (rouge_gemm_i8, quant_int8.cpp:189-211)
//   kind::f8f6f4 e4m3 x e4m3 -> f32 in TMEM          (rouge_gemm_e4m3, fp8.cpp:116-124)
//   kind::f16    f16/bf16 -> f32 in TMEM              (rouge_gemm_f16/bf16, fp16.cpp:123-141)
// and the implicit-GEMM convolution (conv.cpp:26-66, im2col TMA for A).
//
// Two persistent kernels with the same warp roles (384 threads):
//   warp 0      TMA producer: A and B k-blocks into a STAGES-deep ring of
//               128-byte-swizzled shared-memory stages (mbarrier full/empty)
//   warp 1      MMA issuer: one thread issues tcgen05.mma (K = 32 bytes per
//               instruction) into a TMEM accumulator and releases each
//               stage with tcgen05.commit
//   warp 2      TMEM allocator (2 x BN columns: double-buffered accumulator)
//   warps 4-11  epilogue: tcgen05.ld of TMEM lanes, fused scale / dequant /
//               bias / bf16 conversion, TMA tile stores; runs while the MMA
//               warp fills the other accumulator
// gemm_tc_kernel: one CTA per SM, 128 x BN tiles (M = 128 MMAs).
// gemm_tc2_kernel: 2-CTA clusters, 256 x 256 tiles (cta_group::2, M = 256
// MMAs issued by the leader CTA over both CTAs' shared memory and TMEM).
// Tiles are walked in groups of 16 M-blocks so that the CTAs of one wave
// share A and B panels in L2.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <cstring>

#include "formats.cuh"
#include "x86fp.cuh"
#include "ptx.cuh"
#include "i8code.cuh"
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
  const float *scales_a;  // int8: per-row or single scale; MXF8: A's scale atoms (bytes)
  const float *scales_b;  // int8: per-column or single scale; MXF8: B's scale atoms
  int a_rows, b_cols;
  const float *scale_a;   // e4m3 / f16: per-tensor scale scalars (or null)
  const float *scale_b;
  int bf16;               // kind::f16 inputs are bf16
  int use_tma_store;      // C and ldc are 16-byte aligned: epilogue stores through TMA
  int vec16;              // scales_b / bias are 16-byte aligned: vector loads of 4 columns
  int *err;
  // Broadcast output (the sharded W8A8 GEMM): instead of C, every output
  // element goes to column col_off + n of row m of each rank's [M][bld]
  // output, through one multimem store to the multicast address `bcast`
  // (NVLink multicast: the switch writes every bound GPU's copy) or, when
  // bcast is null, through one TMA tile store per entry of peers[0..npeers)
  // (OutMaps built over each rank's block).
  void *bcast;
  void *peers[8];
  int npeers;
  int col_off;
  long long bld;
  // BLAS epilogue (f32 or 16-bit output of the f16 / tf32 / e4m3 kinds,
  // blas != 0): C = alpha * acc + beta * C; the old C is read only when
  // beta != 0.
  int blas;
  float alpha, beta;
  // 16-bit output (OUT_BF16 template) holds IEEE half instead of bf16
  // (cuDNN HALF tensors): hardware round to nearest even.
  int f16out;
  // Implicit-GEMM convolution (A gathered by im2col TMA): M = N*OH*OW
  // output pixels, K = KH*KW*Cin ordered (kr, kc, c), k-block = one filter
  // tap x 64 channels.
  const float *bias;      // per output channel (column) bias added in the epilogue, or null
  int conv_cblocks;       // Cin / 64
  int conv_kw, conv_oh, conv_ow, conv_stride, conv_pad, conv_cin;
  // CTA-pair kernel, last partial round: units from split_from on are the
  // remaining tiles cut N-wise into `split` parts of BN / split columns
  // (one unit per part), so that the round's units fill more clusters.
  int split_from, split;
  // Block-scaled kind (MXF8): operand formats (E4M3 0, E5M2 1) and the
  // number of 128-K blocks per row of the scale-atom arrays.
  int mx_fmt_a, mx_fmt_b, sf_kblocks;
  // Fused per-row quantization of A (the W8A8 linear step, CTA-pair int8
  // kernel only): the launch itself turns the f32 rows fq_x[M][K] into A's
  // codes fq_codes[M][K] and scales fq_scales[M] (= scales_a). fq_cnt[b]
  // counts the finished rows of 128-row block b, fq_cnt[nblk] the finished
  // CTAs and fq_cnt[nblk + 1] the rows handed out (nblk = ceil(M/128)); the
  // last CTA zeroes them all. Rows below fq_rows0 (those of the first round
  // of tiles) are quantized by every warp before the tiles start, the
  // others, in order, by warps 2-3 and by idle epilogue warps while the
  // tiles run.
  const float *fq_x;
  int8_t *fq_codes;
  float *fq_scales;
  unsigned *fq_cnt;
  int fq_rows0;
  // units walk N first (m-block = tile / num_n), so that the first round
  // needs few blocks of A rows
  int n_fast;
  // Batched GEMM with K-major B (item_m > 0): M / item_m items stacked by
  // rows; item i multiplies A rows [i*item_m, +item_m) by B rows
  // [i*N, +N) into C rows [i*item_m, +item_m). item_m is a multiple of
  // 256, so no tile spans two items.
  int item_m;
  // Tile shape of this call (kTileHint*): 0 follows the process-wide
  // rouge_b200_set_tile_mode; the others fix it for this call only (the
  // RougeGemmConfig of the drop-in float GEMMs).
  int tile_hint;
  // Clock probe (rouge_b200_set_clock_probe): CTA b < clk_n writes
  // %clock64 and %globaltimer at its start to clk[4b], clk[4b + 1] and at
  // its end to clk[4b + 2], clk[4b + 3]. Null: no stamps.
  unsigned long long *clk;
  int clk_n;
};

__device__ __forceinline__ void clock_stamp(const GemmArgs &args, int slot) {
  if (args.clk && static_cast<int>(blockIdx.x) < args.clk_n) {
    unsigned long long c;
    asm volatile("mov.u64 %0, %%clock64;" : "=l"(c));
    args.clk[4 * blockIdx.x + slot] = c;
    args.clk[4 * blockIdx.x + slot + 1] = global_timer_ns();
  }
}

constexpr int kTileHintAuto = 0;
constexpr int kTileHintSingle128 = 1;  // one CTA per 128 x 128 tile
constexpr int kTileHintSingle256 = 2;  // one CTA per 128 x 256 tile
constexpr int kTileHintPair = 3;       // CTA pairs, 256 x 256 tiles

constexpr int kStageBytes = 4096;  // one epilogue staging buffer (32 rows x 128 B)

// Output tensor maps of the epilogue's TMA stores: one (this GPU's C), or
// one per rank when the output is broadcast through peer pointers (each
// map covers that rank's copy of this GEMM's column block).
constexpr int kMaxOutMaps = 8;
struct alignas(64) OutMaps {
  CUtensorMap m[kMaxOutMaps];
  // Block-scaled kind: scale-factor atoms of A and B (rows of 128 bytes,
  // four rows = one 512-byte atom of 128 rows x 4 K-blocks).
  CUtensorMap sfa, sfb;
  int n;
};

template <MmaKind KIND, int BN, bool B_MN>
struct Cfg {
  static constexpr int ESIZE = KIND == MmaKind::TF32 ? 4 : (KIND == MmaKind::F16 ? 2 : 1);
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

// Unit u of the CTA-pair kernel: tile (mb, nb), part `part` of `parts`.
__device__ __forceinline__ void unit_coords(int u, const GemmArgs &args, int &mb, int &nb, int &part,
                                            int &parts) {
  int t = u;
  part = 0;
  parts = 1;
  if (u >= args.split_from) {
    parts = args.split;
    t = args.split_from + (u - args.split_from) / parts;
    part = (u - args.split_from) - (t - args.split_from) * parts;
  }
  if (args.n_fast) {
    mb = t / args.num_n;
    nb = t - mb * args.num_n;
  } else {
    tile_coords(t, args.num_m, args.num_n, mb, nb);
  }
}

__device__ __forceinline__ void report(int *err, volatile int *abort, int code) {
  *abort = 1;
  if (err) atomicCAS(err, 0, code);
}

// 32 consecutive f32 values of a per-column vector (column scales, bias)
// starting at column col0, identical in every lane: eight 16-byte loads of
// one address per warp (broadcast) when the chunk is whole and the vector
// 16-byte aligned, else one element per lane and shuffles.
__device__ __forceinline__ void column_vector(const float *vec, bool vec16, int col0, int N,
                                              int lane, float (&out)[32]) {
  if (vec16 && col0 + 32 <= N) {
    const float4 *p = reinterpret_cast<const float4 *>(vec + col0);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float4 t = __ldg(p + q);
      out[4 * q] = t.x;
      out[4 * q + 1] = t.y;
      out[4 * q + 2] = t.z;
      out[4 * q + 3] = t.w;
    }
  } else {
    const int col = col0 + lane;
    const float mine = col < N ? __ldg(vec + col) : 0.0f;
#pragma unroll
    for (int j = 0; j < 32; ++j) out[j] = __shfl_sync(0xffffffffu, mine, j);
  }
}

// Component k of a float4 (k a compile-time constant after unrolling).
__device__ __forceinline__ float f4_at(const float4 &v, int k) {
  return k == 0 ? v.x : (k == 1 ? v.y : (k == 2 ? v.z : v.w));
}

// The warp's per-column vector (column scales, bias) prefetched once per
// tile: lane l holds columns 4l .. 4l + 3 from the warp's first column; the
// 32 values of chunk c come from lanes 8c .. 8c + 7 by shuffles.
struct ColVec {
  float4 v;
  bool on;  // prefetched (else column_vector per chunk)
  bool ok;  // every column scale and the rows' scales finite and below 2^96
};

// Converts one 32-column chunk of one warp's 32 accumulator rows (thread =
// row, v[j] = column col0 + j) and writes it to C.
//   TMA path: the chunk goes to a 128-byte (f32/i32) or 64-byte (bf16)
//   swizzled staging buffer `buf` in shared memory and one lane issues a
//   tiled TMA store of the 32 x 32 box; out-of-range rows and columns are
//   clipped by the tensor map. With NBUF staging buffers per warp used in
//   turn, the store of the previous NBUF - 1 chunks may still be reading.
//   Direct path (C not 16-byte aligned): predicated per-thread stores.
template <MmaKind KIND, int OUT, int NBUF>
__device__ __forceinline__ void epilogue_chunk(const GemmArgs &args, const uint32_t (&v)[32],
                                               int col0, int row0, int row, bool row_ok, float sa,
                                               bool sa_ok, float sab, uint8_t *buf,
                                               const OutMaps *om, int lane, const ColVec &cv,
                                               int cv_lane) {
  uint32_t o[32];  // f32 / i32 bits, or bf16 pairs in o[0..15]
  // this chunk's 32 column values from the tile's prefetch
  auto col_values = [&](float (&out)[32]) {
#pragma unroll
    for (int j = 0; j < 32; ++j) out[j] = __shfl_sync(0xffffffffu, f4_at(cv.v, j & 3), cv_lane + (j >> 2));
  };
  if constexpr (OUT == ROUGE_B200_OUT_I32) {
#pragma unroll
    for (int j = 0; j < 32; ++j) o[j] = v[j];
  } else {
    float f[32];
    bool may_nan = true;
    if constexpr (KIND == MmaKind::I8) {
      // quant_int8.cpp:208: ((float)acc * sa) * sb, two rounded multiplies.
      // With sa and every column scale of the chunk finite and below 2^96,
      // (float)acc * sa is finite (|acc| < 2^31) and the second product can
      // only overflow to +-inf, which x86 and the GPU both produce: no NaN,
      // so plain (paired) multiplies are exact here.
      float sb[32];
      bool fast;
      if (cv.on) {
        col_values(sb);
        fast = cv.ok;
      } else {
        const int col = col0 + lane;
        const float sbl = args.b_cols ? (col < args.N ? __ldg(args.scales_b + col) : 0.0f)
                                      : __ldg(args.scales_b);
        fast = __all_sync(0xffffffffu, sa_ok && fabsf(sbl) < 7.9e28f);
        if (args.b_cols) {
          column_vector(args.scales_b, args.vec16, col0, args.N, lane, sb);
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) sb[j] = sbl;
        }
      }
      may_nan = !fast;
      if (fast) {
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          float a0 = __int2float_rn(static_cast<int32_t>(v[j]));
          float a1 = __int2float_rn(static_cast<int32_t>(v[j + 1]));
          mul2(a0, a1, a0, a1, sa);
          mul2(f[j], f[j + 1], a0, a1, sb[j], sb[j + 1]);
        }
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          f[j] = x86_mul(x86_mul(__int2float_rn(static_cast<int32_t>(v[j])), sa), sb[j]);
      }
    } else if (args.bias) {
      // conv.cpp:61-64: bias added to the finished f32 sum of each channel
      float bv[32];
      if (cv.on)
        col_values(bv);
      else
        column_vector(args.bias, args.vec16, col0, args.N, lane, bv);
#pragma unroll
      for (int j = 0; j < 32; j += 2)
        add2(f[j], f[j + 1], __uint_as_float(v[j]), __uint_as_float(v[j + 1]), bv[j], bv[j + 1]);
    } else {
#pragma unroll
      for (int j = 0; j < 32; j += 2)
        mul2(f[j], f[j + 1], __uint_as_float(v[j]), __uint_as_float(v[j + 1]), sab);
    }
    // BLAS form C = alpha * acc + beta * C: sab holds alpha; the old C is
    // read only when beta != 0 (it need not be valid otherwise).
    if constexpr (OUT == ROUGE_B200_OUT_BF16 && KIND != MmaKind::I8) {
      if (args.blas && args.beta != 0.0f && row_ok) {
        const uint16_t *crow =
            static_cast<const uint16_t *>(args.C) + static_cast<long long>(row) * args.ldc;
        const bool whole = col0 + 32 <= args.N && (args.ldc % 8) == 0 &&
                           (reinterpret_cast<uintptr_t>(args.C) & 15u) == 0;
#pragma unroll
        for (int j = 0; j < 32; j += 8) {
          uint32_t h[4];
          if (whole) {
            const uint4 t = *reinterpret_cast<const uint4 *>(crow + col0 + j);
            h[0] = t.x; h[1] = t.y; h[2] = t.z; h[3] = t.w;
          } else {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const int c = col0 + j + 2 * q;
              h[q] = (c < args.N ? crow[c] : 0u) | ((c + 1 < args.N ? crow[c + 1] : 0u) << 16);
            }
          }
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const uint32_t bits = (h[q >> 1] >> ((q & 1) * 16)) & 0xFFFFu;
            const float c = args.f16out ? __half2float(__ushort_as_half(static_cast<unsigned short>(bits)))
                                        : __uint_as_float(bits << 16);
            f[j + q] = __fmaf_rn(args.beta, c, f[j + q]);
          }
        }
      }
    }
    if constexpr (OUT == ROUGE_B200_OUT_F32 && KIND != MmaKind::I8) {
      if (args.blas && args.beta != 0.0f && row_ok) {
        const float *crow = static_cast<const float *>(args.C) + static_cast<long long>(row) * args.ldc;
        const bool whole = col0 + 32 <= args.N && (args.ldc % 4) == 0 &&
                           (reinterpret_cast<uintptr_t>(args.C) & 15u) == 0;
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          float c4[4];
          if (whole) {
            const float4 t = *reinterpret_cast<const float4 *>(crow + col0 + j);
            c4[0] = t.x; c4[1] = t.y; c4[2] = t.z; c4[3] = t.w;
          } else {
#pragma unroll
            for (int q = 0; q < 4; ++q) c4[q] = col0 + j + q < args.N ? crow[col0 + j + q] : 0.0f;
          }
#pragma unroll
          for (int q = 0; q < 4; ++q) f[j + q] = __fmaf_rn(args.beta, c4[q], f[j + q]);
        }
      }
    }
    if constexpr (OUT == ROUGE_B200_OUT_F32) {
#pragma unroll
      for (int j = 0; j < 32; ++j) o[j] = __float_as_uint(f[j]);
    } else if (args.f16out) {
#pragma unroll
      for (int j = 0; j < 16; ++j) o[j] = f16x2_rn(f[2 * j], f[2 * j + 1]);
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

  if (args.bcast || (OUT == ROUGE_B200_OUT_BF16 && args.npeers)) {
    // Stage the chunk as row `lane` of the warp's line buffer: 32 rows of
    // 128 bytes (one 64-column bf16 line, chunk pairs in its two halves, or
    // one 32-column f32 line), 16-byte units XOR-swizzled by row -- the
    // layout of a 128-byte-swizzled TMA box. bcast_flush writes the buffer
    // out along rows to the multicast address; peer_flush stores it as one
    // 64 x 32 box into every rank's C.
    constexpr int kUnits = OUT == ROUGE_B200_OUT_BF16 ? 4 : 8;
    const int ubase = OUT == ROUGE_B200_OUT_BF16 ? ((col0 >> 5) & 1) * 4 : 0;
    if (!args.bcast && ubase == 0) {  // a new line: the last line's stores have read the buffer
      if (lane == 0) bulk_wait_read<0>();
      __syncwarp();
    }
    const uint32_t rbase = smem_u32(buf) + static_cast<uint32_t>(lane) * 128u;
#pragma unroll
    for (int q = 0; q < kUnits; ++q)
      st_shared_v4(rbase + ((static_cast<uint32_t>(ubase + q) ^ (static_cast<uint32_t>(lane) & 7u)) << 4),
                   o[4 * q], o[4 * q + 1], o[4 * q + 2], o[4 * q + 3]);
    return;
  }

  if (args.use_tma_store) {
    if (lane == 0) bulk_wait_read<NBUF - 1>();  // this buffer's previous store has read it
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
      if (row0 < args.M)
        for (int r = 0; r < om->n; ++r) tma_store_2d(&om->m[r], buf, col0, row0);
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

// Writes the warp's staged line buffer (see epilogue_chunk) to the
// multicast address: line_col0 = first column of the 128-byte line,
// `units` = mask of the staged 16-byte units. Each store instruction covers
// 4 rows x 128 contiguous bytes (8 lanes per row).
template <int OUT>
__device__ __forceinline__ void bcast_flush(const GemmArgs &args, const uint8_t *buf, int row0,
                                            int line_col0, uint32_t units, int lane) {
  constexpr int kEpu = OUT == ROUGE_B200_OUT_BF16 ? 8 : 4;  // elements per 16-byte unit
  constexpr size_t kEsz = OUT == ROUGE_B200_OUT_BF16 ? 2 : 4;
  __syncwarp();
  const int u = lane & 7;
  const bool unit_ok = ((units >> u) & 1u) && line_col0 + u * kEpu < args.N;
#pragma unroll
  for (int it = 0; it < 8; ++it) {
    const int r = it * 4 + (lane >> 3);
    if (unit_ok && row0 + r < args.M) {
      const uint4 v = ld_shared_v4(smem_u32(buf) + static_cast<uint32_t>(r) * 128u +
                                   ((static_cast<uint32_t>(u) ^ (static_cast<uint32_t>(r) & 7u)) << 4));
      const size_t off = (static_cast<size_t>(row0 + r) * args.bld +
                          static_cast<size_t>(args.col_off + line_col0 + u * kEpu)) * kEsz;
      multimem_st_v4(reinterpret_cast<uint64_t>(args.bcast) + off, v);
    }
  }
  __syncwarp();
}

// Stores the warp's staged 64-column bf16 line (see epilogue_chunk) into
// every rank's C: one 64 x 32 TMA box per rank (128-byte rows), clipped at
// the M and N edges by the tensor maps.
__device__ __forceinline__ void peer_flush(const uint8_t *buf, const OutMaps *om, int row0,
                                           int line_col0, int M, int lane) {
  fence_async_smem();
  __syncwarp();
  if (lane == 0) {
    if (row0 < M)
      for (int r = 0; r < om->n; ++r) tma_store_2d(&om->m[r], buf, line_col0, row0);
    bulk_commit();
  }
}

// One epilogue warp's share of one accumulator tile of `width` columns
// (C columns col0 ..) held from TMEM column tcol: TMEM lanes
// [32*quarter, +32) (C rows m0 + 32*quarter + lane) and column half `half`.
// Two 32-column tcgen05.ld loads are kept in flight: chunk c+1 loads while
// chunk c is converted and stored.
// Overlapping accumulator buffers (ovl_bar != 0): the warps of column half
// ovl_half arrive on ovl_bar (a cluster address) once per tile: right after
// reading chunk ovl_chunk (the chunk shared with the other buffer, which
// they read first), or at once when the tile does not hold it (ovl_chunk
// < 0) or it lies past N.
template <MmaKind KIND, int OUT, int NBUF>
__device__ __forceinline__ void epilogue_tile(const GemmArgs &args, uint32_t tcol, int m0, int col0,
                                              int width, int quarter, int half, float sab,
                                              uint8_t *stage, int &seq, const OutMaps *om,
                                              int lane, uint32_t ovl_bar = 0u, int ovl_half = 0,
                                              int ovl_chunk = -1, int ovl_count = 1) {
  const int row0 = m0 + quarter * 32;
  const int row = row0 + lane;
  const bool row_ok = row < args.M;
  float sa = 1.0f;
  if constexpr (KIND == MmaKind::I8) {
    // (scales written by this launch itself are read through L2)
    if (OUT != ROUGE_B200_OUT_I32 && row_ok)
      sa = args.fq_cnt ? __ldcg(args.scales_a + row) : __ldg(args.scales_a + (args.a_rows ? row : 0));
  }
  const bool sa_ok = fabsf(sa) < 7.9e28f;  // finite and below 2^96
  const uint32_t tbase = tcol + (static_cast<uint32_t>(quarter * 32) << 16);
  const int cols_left = args.N - col0;
  const int nchunks = cols_left >= width ? width / 32 : (cols_left + 31) / 32;  // warp-uniform
  const int per_half = width >= 64 ? width / 64 : 1;  // (a 32-wide tile: the first half's warps)
  const int c_end = min(nchunks, (half + 1) * per_half);
  const int c_beg = half * per_half;
  // The fused W8A8 step's column scales: one load per tile instead of one
  // L2 round trip per chunk (16-byte aligned vectors; the warp's first
  // column is a multiple of 32). The fast-path test covers all of the
  // warp's columns at once; a chunk it sends to the exact path gets the
  // same values. (The step measured 0.6 % faster with it; the plain GEMMs
  // and the convolution, with the same loads for their scales or bias,
  // 0.4-0.5 % slower, so they keep the per-chunk loads.)
  ColVec cv;
  const float *cvec = KIND == MmaKind::I8 ? (args.b_cols ? args.scales_b : nullptr) : args.bias;
  cv.on = OUT != ROUGE_B200_OUT_I32 && cvec != nullptr && args.vec16 && c_beg < c_end &&
          args.fq_cnt != nullptr;
  cv.v = make_float4(0.f, 0.f, 0.f, 0.f);
  cv.ok = false;
  if (cv.on) {
    const int c = col0 + c_beg * 32 + 4 * lane;
    if (c + 3 < args.N) {
      cv.v = __ldg(reinterpret_cast<const float4 *>(cvec + c));
    } else {
      cv.v.x = c < args.N ? __ldg(cvec + c) : 0.0f;
      cv.v.y = c + 1 < args.N ? __ldg(cvec + c + 1) : 0.0f;
      cv.v.z = c + 2 < args.N ? __ldg(cvec + c + 2) : 0.0f;
    }
    if constexpr (KIND == MmaKind::I8) {
      const float m = fmaxf(fmaxf(fabsf(cv.v.x), fabsf(cv.v.y)), fmaxf(fabsf(cv.v.z), fabsf(cv.v.w)));
      cv.ok = __all_sync(0xffffffffu, sa_ok && m < 7.9e28f);  // (a NaN fails the compare)
    }
  }
  const bool ovl = ovl_bar != 0u && half == ovl_half;
  // shared chunks this warp reads (they lead the order; the arrival follows
  // the last of them)
  const int ovl_n = (ovl && ovl_chunk >= c_beg && ovl_chunk < c_end)
                        ? min(ovl_count, c_end - ovl_chunk) : 0;
  auto ovl_done = [&]() {
    tc_fence_before_sync();
    __syncwarp();
    if (lane == 0) mbar_arrive_cluster(ovl_bar);
  };
  if (ovl && ovl_n == 0) ovl_done();  // nothing of the shared chunks is read
  if (c_beg >= c_end) return;
  const int nrot = c_end - c_beg;
  const int rot = ovl_n ? ovl_chunk - c_beg : 0;
  auto chunk = [&](int j) {
    const int k = j + rot;
    return c_beg + (k >= nrot ? k - nrot : k);
  };
  uint32_t va[32], vb[32];
  tmem_ld_32x32b_x32(tbase + static_cast<uint32_t>(chunk(0) * 32), va);
  tmem_ld_wait_regs(va);
  int loaded = 1;
  if (ovl_n == 1) ovl_done();
  // staging buffer of this warp's seq-th chunk (the multicast output stages
  // whole lines in the first buffer)
  const bool lines = args.bcast || (OUT == ROUGE_B200_OUT_BF16 && args.npeers);
  auto buf = [&]() {
    return lines ? stage : stage + (NBUF > 1 ? (seq++ & 1) * kStageBytes : 0);
  };
  // multicast or peer-store output: flush after chunk c when its line is
  // complete
  uint32_t staged = 0;
  auto after = [&](int c) {
    if (!lines) return;
    const int cc = col0 + c * 32;
    if (OUT == ROUGE_B200_OUT_BF16) {
      staged |= ((cc >> 5) & 1) ? 0xF0u : 0x0Fu;
      if (((cc >> 5) & 1) || c + 1 == c_end) {
        if (args.bcast)
          bcast_flush<OUT>(args, stage, row0, cc & ~63, staged, lane);
        else
          peer_flush(stage, om, row0, cc & ~63, args.M, lane);
        staged = 0;
      }
    } else {
      bcast_flush<OUT>(args, stage, row0, cc, 0xFFu, lane);
    }
  };
  // (a rotated order only occurs without multicast output, whose line
  // flushes assume ascending chunks)
  for (int j = 0; j < nrot; j += 2) {
    if (j + 1 < nrot) tmem_ld_32x32b_x32(tbase + static_cast<uint32_t>(chunk(j + 1) * 32), vb);
    epilogue_chunk<KIND, OUT, NBUF>(args, va, col0 + chunk(j) * 32, row0, row, row_ok, sa, sa_ok,
                                    sab, buf(), om, lane, cv, (chunk(j) - c_beg) * 8);
    after(chunk(j));
    if (j + 1 < nrot) {
      tmem_ld_wait_regs(vb);
      if (++loaded == ovl_n) ovl_done();
      if (j + 2 < nrot) tmem_ld_32x32b_x32(tbase + static_cast<uint32_t>(chunk(j + 2) * 32), va);
      epilogue_chunk<KIND, OUT, NBUF>(args, vb, col0 + chunk(j + 1) * 32, row0, row, row_ok, sa,
                                      sa_ok, sab, buf(), om, lane, cv, (chunk(j + 1) - c_beg) * 8);
      after(chunk(j + 1));
      if (j + 2 < nrot) {
        tmem_ld_wait_regs(va);
        if (++loaded == ovl_n) ovl_done();
      }
    }
  }
}

// Convolution: im2col box position (w, h, image) of output pixel p0, the
// first pixel of a 128-row A block.
__device__ __forceinline__ void conv_box(const GemmArgs &args, int p0, int &cw, int &ch, int &cn) {
  const int ohw = args.conv_oh * args.conv_ow;
  cn = p0 / ohw;
  const int rem = p0 - cn * ohw;
  ch = (rem / args.conv_ow) * args.conv_stride - args.conv_pad;
  cw = (rem % args.conv_ow) * args.conv_stride - args.conv_pad;
}

// K-block kb of a convolution: filter tap (kr, kc), first channel c0, and
// the K coordinate of the matching weight columns.
__device__ __forceinline__ void conv_kblock(const GemmArgs &args, int kb, int bk, int &c0, int &kr,
                                            int &kc, int &kx) {
  const int tap = kb / args.conv_cblocks;
  c0 = (kb - tap * args.conv_cblocks) * bk;
  kr = tap / args.conv_kw;
  kc = tap - kr * args.conv_kw;
  kx = tap * args.conv_cin + c0;
}

template <MmaKind KIND, int BN, bool B_MN, int OUT, bool CONV = false>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ OutMaps om, const GemmArgs args) {
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

  if (threadIdx.x == 0) clock_stamp(args, 0);
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
  // Everything above overlaps the previous kernel's tail when this launch
  // is programmatically serialised; its outputs (A, the scales) are read
  // only after this point.
  grid_dependency_wait();
  // The next programmatically serialised launch may start its own set-up
  // on SMs this grid leaves (its CTAs then wait for this grid to complete).
  grid_launch_dependents();

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ producer
    int it = 0;
    bool ok = true;
    for (int t = blockIdx.x; ok && t < args.num_tiles; t += gridDim.x) {
      int mb, nb;
      tile_coords(t, args.num_m, args.num_n, mb, nb);
      int cw = 0, ch = 0, cn = 0;
      if constexpr (CONV) conv_box(args, mb * kBM, cw, ch, cn);
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
          int c0, kr, kc;
          conv_kblock(args, kb, C::BK, c0, kr, kc, kx);
          tma_load_im2col_4d(sA + s * C::A_BYTES, &tmA, &full[s], c0, cw, ch, cn,
                             static_cast<uint16_t>(kc), static_cast<uint16_t>(kr));
        } else {
          tma_load_2d(sA + s * C::A_BYTES, &tmA, &full[s], kx, mb * kBM);
        }
        if constexpr (!B_MN) {
          tma_load_2d(sB + s * C::B_BYTES, &tmB, &full[s], kx,
                      nb * BN + (args.item_m ? (mb * kBM / args.item_m) * args.N : 0));
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
    // S8 (1) / E4M3 (0) / F16 (0) / TF32 (2); BF16 (1) below
    constexpr uint32_t ab_fmt = KIND == MmaKind::I8 ? 1u : (KIND == MmaKind::TF32 ? 2u : 0u);
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
    int local = 0, seq = 0;
    float sab = 1.0f;
    if constexpr (KIND != MmaKind::I8) {
      if (args.scale_a && args.scale_b) sab = x86_mul(__ldg(args.scale_a), __ldg(args.scale_b));
      if (args.blas) sab = args.alpha;
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
      epilogue_tile<KIND, OUT, 1>(args, tmem_base + static_cast<uint32_t>(slot * BN), mb * kBM,
                                  nb * BN, BN, quarter, half, sab, stage, seq, &om, lane);
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[slot]);
    }
    if (args.use_tma_store && lane == 0) bulk_wait_all();
    // Broadcast stores reach other GPUs: order them before anything this
    // thread's kernel completion releases (the cross-rank barrier after it).
    if (args.bcast || args.npeers) asm volatile("fence.acq_rel.sys;" ::: "memory");
  }

  tc_fence_before_sync();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after_sync();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
  if (threadIdx.x == 0) clock_stamp(args, 2);
}

// ----------------------------------------------------------- CTA-pair tiles
//
// A 2-CTA cluster computes a 256 x BN tile with tcgen05.mma.cta_group::2
// (M = 256): CTA rank r loads rows [128r, +128) of the A block and half r
// of B's BN rows/columns into its own stage ring, the leader (rank 0) issues
// the MMAs for both, and each CTA's TMEM receives its own 128 accumulator
// rows, which its own epilogue warps drain. Per 128 x BN of output each SM
// thus reads 128 + BN/2 operand rows from shared memory instead of 128 + BN:
// the operand feed, not the tensor pipe, limits the single-CTA tile.
//
// Synchronisation (all barriers live in the CTA that waits on them):
//   full[s]   leader only: armed by the leader's producer with both CTAs'
//             bytes; both producers' loads complete_tx on it (cta_group::2
//             TMA form, barrier addressed in the leader)
//   empty[s]  each CTA: the leader's MMA commit arrives on both
//   tfull[2]  each CTA: the leader's commit after a tile's last k-block
//   tempty[2] leader only: 16 arrivals, one per epilogue warp of each CTA
template <MmaKind KIND, int BN, bool B_MN, bool FQ = false>
struct Cfg2 {
  static constexpr int ESIZE = KIND == MmaKind::TF32 ? 4 : (KIND == MmaKind::F16 ? 2 : 1);
  static constexpr int BK = kBKBytes / ESIZE;
  static constexpr int UMMA_K = 32 / ESIZE;
  static constexpr int HALF_N = BN / 2;  // B rows (K-major) / columns (MN-major) per CTA
  static constexpr int A_BYTES = kBM * kBKBytes;
  static constexpr int B_BYTES = HALF_N * kBKBytes;
  // Block-scaled kind: per stage the scale atoms of this CTA's 128 A rows
  // and of all BN B rows (each CTA's TMEM needs the scales of every B row).
  // block-scaled kinds: one 512-byte scale atom (128 rows x 4 scales) per
  // 128 rows per ATOMS_K: MXF8 one per stage (4 K-blocks of 32 = the
  // stage's 128 K), NVF4 four (one per MMA: 4 blocks of 16 = 64 K)
  // (MXF4: two per 128 rows, 8 blocks of 32 = the stage's 256 K)
  static constexpr bool NV = KIND == MmaKind::NVF4;
  static constexpr bool F4 = KIND == MmaKind::MXF4;
  static constexpr bool MX = KIND == MmaKind::MXF8 || NV || F4;
  static constexpr int ATOMS_K = NV ? 4 : (F4 ? 2 : 1);
  static constexpr int SFA_BYTES = MX ? ATOMS_K * 512 : 0;
  static constexpr int SFB_BYTES = MX ? (BN / 128) * ATOMS_K * 512 : 0;
  // per-stage scale region, padded so that stages stay 1024-byte multiples
  static constexpr int SF_STAGE = MX ? (SFA_BYTES + SFB_BYTES + 1023) / 1024 * 1024 : 0;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES + SF_STAGE;
  // TMEM: accumulator buffer 0 at column 0, buffer 1 at ACC1_COL, then
  // SF_BUFS rotating sets of scale words (SFA: 4 columns, SFB: 4 columns
  // per 128 B rows). A 256-wide block-scaled tile leaves no room for two
  // disjoint buffers and the scales: its buffers overlap in 32 columns
  // (buffer 0's last chunk is buffer 1's first), which each tile's
  // epilogue drains first and reports on its own barrier.
  static constexpr int SF_SET = ATOMS_K * (4 + BN / 32);  // MXF8 12, MXF4 24, NVF4 48 (BN 256)
  static constexpr int SF_COL = MX && BN == 256 ? (NV ? 448 : 480) : 2 * BN;
  static constexpr int SF_BUFS = MX && BN == 256 ? (NV || F4 ? 1 : 2) : (NV ? 1 : 4);
  static constexpr int ACC1_COL = MX && BN == 256 ? SF_COL - BN : BN;
  static constexpr int OVL_CHUNKS = (BN - ACC1_COL) / 32;  // chunks both buffers share
  static constexpr bool OVERLAP = OVL_CHUNKS > 0;
  static_assert(OVL_CHUNKS <= 2 && (BN - ACC1_COL) % 32 == 0, "shared chunks");
  static constexpr int TMEM_COLS = MX ? 512 : 2 * BN;
  static constexpr int B_CHUNKS = (HALF_N * ESIZE) / kBKBytes;
  static constexpr int B_CHUNK_BYTES = B_MN ? BK * kBKBytes : B_BYTES;
  // fused quantization: the prologue's 12 row slots of 16 KB (one per
  // warp) are stage memory, so the kernel keeps 6 stages; 12 more
  // mbarriers (one per warp's row slot)
  static constexpr int QSLOT = 16384;
  static constexpr int BAR_BYTES = FQ ? 512 : 256;
#ifndef RB200_PAIR_EPI_BUFS  // staging buffers per epilogue warp (tuning builds)
#define RB200_PAIR_EPI_BUFS 1
#endif
  static constexpr int EPI_BUFS = RB200_PAIR_EPI_BUFS;
  static constexpr int EPI_BYTES = 8 * EPI_BUFS * kStageBytes;
  static constexpr int STAGE_ROOM =
      (232448 - 1024 - EPI_BYTES - BAR_BYTES) / STAGE_BYTES;
#ifdef RB200_PAIR_STAGES  // stage-count override for tuning builds
  static constexpr int STAGES = RB200_PAIR_STAGES;
#else
  static constexpr int STAGES = STAGE_ROOM > 8 ? 8 : STAGE_ROOM;
#endif
  static constexpr int BAR_OFF = STAGES * STAGE_BYTES + EPI_BYTES;
  static constexpr int SMEM = 1024 + BAR_OFF + BAR_BYTES;
  static_assert(SMEM <= 232448, "exceeds the 227 KB per-CTA shared memory limit");
  static_assert(STAGE_BYTES % 1024 == 0, "stages keep the 1024-byte swizzle alignment");
  // the prologue's 12 row slots, all in stage memory
  static_assert(!FQ || (KIND == MmaKind::I8 && STAGES * STAGE_BYTES >= 12 * QSLOT), "FQ");
  static_assert(BN % 32 == 0 && BN >= 64 && BN <= 256, "BN");
  static_assert(!B_MN || B_CHUNKS >= 1, "MN-major B needs whole 128-byte chunks per CTA");
  static_assert(TMEM_COLS == 128 || TMEM_COLS == 256 || TMEM_COLS == 512, "TMEM columns");
  static_assert(ACC1_COL + BN <= (MX ? SF_COL : TMEM_COLS), "accumulators below the scales");
  static_assert(!MX || (BN % 128 == 0 && !B_MN && SF_COL + SF_BUFS * SF_SET <= TMEM_COLS),
                "MX tile");
};

// Rows of the fused quantizer claimed while the tiles run get an L2
// prefetch this many rows ahead of the row claimed.
constexpr int kFqAhead = 512;

// Scale and codes of one row held in registers (v[j] = float4 j * 32 +
// lane of the row; nvec float4 in all) as quant_int8.cpp:72-90 computes
// them: scale and reciprocal in double, branch-free single-precision codes,
// words near a rounding tie re-encoded in double afterwards from a second
// read of their inputs (xr). Then one count on the row's 128-row block
// (release: the codes and scale are visible to whoever sees the count).
template <int VPL>
__device__ __forceinline__ void fq_encode_row(const GemmArgs &args, int r, const float4 (&v)[VPL],
                                              int nvec, int lane) {
  float amax = 0.0f;
#pragma unroll
  for (int j = 0; j < VPL; ++j)
    amax = max3(amax, max3(fabsf(v[j].x), fabsf(v[j].y), fabsf(v[j].z)), fabsf(v[j].w));
#pragma unroll
  for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const double a = static_cast<double>(amax);
  const float sc = a > 0.0 ? __double2float_rn(__ddiv_rn(a, 127.0)) : 1.0f;
  const double inv = __ddiv_rn(1.0, static_cast<double>(sc));
  const float inv_f = __double2float_rn(inv);
  const bool exact_row = isinf(inv_f);
  if (lane == 0) args.fq_scales[r] = sc;
  uint32_t *orow = reinterpret_cast<uint32_t *>(args.fq_codes + static_cast<size_t>(r) * args.K);
  uint32_t redo = 0;
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    const int i = j * 32 + lane;
    bool tie;
    const uint32_t w = encode4_i8_fast(v[j], inv_f, tie);
    tie |= exact_row;
    if (i < nvec && !tie) orow[i] = w;
    redo |= (tie && i < nvec) ? (1u << j) : 0u;
  }
  const float4 *xr = reinterpret_cast<const float4 *>(args.fq_x + static_cast<size_t>(r) * args.K);
  while (redo) {
    const int j = __ffs(redo) - 1;
    redo &= redo - 1;
    orow[j * 32 + lane] = encode4_i8_exact(__ldg(xr + j * 32 + lane), inv);
  }
  // codes and scale before the count, also for the TMA loads that read them
  fence_async_global();
  __syncwarp();
  if (lane == 0) red_release_add(args.fq_cnt + (r >> 7), 1u);
}

// Rows [0, fq_rows0) of the fused quantizer (GemmArgs::fq_x), before the
// tiles start: every warp of the grid takes rows with the stride of the
// grid's warps (12 per CTA) through its 16 KB shared-memory slot -- bulk
// copy, registers (32 float4 per lane: rows up to 4096 elements), the next
// row's copy into the slot, then fq_encode_row. A copy that does not land
// in time reports ROUGE_B200_ETIMEOUT and ends the warp's rows (the block
// counts then stay short and the tiles that need them time out as well).
__device__ __forceinline__ void fq_rows_first(const GemmArgs &args, uint8_t *slot, uint64_t *bar,
                                              int warp, int lane) {
  constexpr int kVpl = 32;
  const int end = args.fq_rows0;
  const int gw = static_cast<int>(gridDim.x) * 12;
  int r = static_cast<int>(blockIdx.x) * 12 + warp;
  const uint32_t row_bytes = static_cast<uint32_t>(args.K) * 4u;
  const int nvec = args.K >> 2;
  bool in_flight = r < end;
  if (lane == 0 && in_flight) {
    mbar_arrive_expect_tx(bar, row_bytes);
    bulk_load(slot, args.fq_x + static_cast<size_t>(r) * args.K, row_bytes, bar);
  }
  const volatile int never = 0;
  uint32_t phase = 0;
  while (r < end) {
    const bool got = mbar_wait(bar, phase, &never);
    if (!__all_sync(0xffffffffu, got)) {
      if (lane == 0 && args.err) atomicCAS(args.err, 0, ROUGE_B200_ETIMEOUT);
      break;
    }
    phase ^= 1u;
    in_flight = false;
    const float4 *row = reinterpret_cast<const float4 *>(slot);
    float4 v[kVpl];
#pragma unroll
    for (int j = 0; j < kVpl; ++j) {
      const int i = j * 32 + lane;
      v[j] = i < nvec ? row[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    // the slot is in registers: it takes the warp's next row
    fence_async_smem();
    __syncwarp();
    const int rn = r + gw;
    if (lane == 0 && rn < end) {
      mbar_arrive_expect_tx(bar, row_bytes);
      bulk_load(slot, args.fq_x + static_cast<size_t>(rn) * args.K, row_bytes, bar);
      in_flight = true;
    }
    fq_encode_row(args, r, v, nvec, lane);
    r = rn;
  }
  if (in_flight && lane == 0) mbar_wait(bar, phase, &never);  // let the last copy land
  // L2 prefetch of the first rows the running tiles' quantizer will claim
  const int pf = args.fq_rows0 + static_cast<int>(blockIdx.x) * 12 + warp;
  if (lane == 0 && pf < args.M && pf < args.fq_rows0 + kFqAhead)
    bulk_prefetch_l2(args.fq_x + static_cast<size_t>(pf) * args.K, row_bytes);
}

// Rows [fq_rows0, M) of the fused quantizer are handed out in order from
// a counter (fq_cnt[nblk + 1]) while the tiles run, to warps 2-3 and to the
// epilogue warps while their next accumulator is not ready. Returns the
// claimed row (>= M: none left) and starts an L2 prefetch of the row
// kFqAhead places further on, which the warps claim a few microseconds
// later; the first kFqAhead rows are prefetched by fq_rows_first.
__device__ __forceinline__ int fq_claim(const GemmArgs &args, int lane) {
  const int nblk = (args.M + kBM - 1) / kBM;
  int r = 0;
  if (lane == 0) {
    r = args.fq_rows0 + static_cast<int>(atomicAdd(args.fq_cnt + nblk + 1, 1u));
    if (r + kFqAhead < args.M)
      bulk_prefetch_l2(args.fq_x + static_cast<size_t>(r + kFqAhead) * args.K,
                       static_cast<uint32_t>(args.K) * 4u);
  }
  return __shfl_sync(0xffffffffu, r, 0);
}

// One claimed row, loaded straight into registers (no shared memory and
// no TMA queue, which the tiles' loads keep busy) in two passes of half a
// row per lane each: the maximum (loads kept in L2), then the codes from a
// second read of the row. Half the registers of a whole row in flight,
// which the epilogue warps that run this between tiles need.
__device__ __forceinline__ void fq_row_direct(const GemmArgs &args, int r, int lane) {
  constexpr int kHalf = 16;  // float4 per lane per pass: rows up to 4096 elements
  const int nvec = args.K >> 2;
  const float4 *xr = reinterpret_cast<const float4 *>(args.fq_x + static_cast<size_t>(r) * args.K);
  float amax = 0.0f;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    float4 v[kHalf];
#pragma unroll
    for (int j = 0; j < kHalf; ++j) {
      const int i = (h * kHalf + j) * 32 + lane;
      v[j] = i < nvec ? __ldcg(xr + i) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int j = 0; j < kHalf; ++j)
      amax = max3(amax, max3(fabsf(v[j].x), fabsf(v[j].y), fabsf(v[j].z)), fabsf(v[j].w));
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  // quant_int8.cpp:82-84: scale and reciprocal in double
  const double a = static_cast<double>(amax);
  const float sc = a > 0.0 ? __double2float_rn(__ddiv_rn(a, 127.0)) : 1.0f;
  const double inv = __ddiv_rn(1.0, static_cast<double>(sc));
  const float inv_f = __double2float_rn(inv);
  const bool exact_row = isinf(inv_f);
  if (lane == 0) args.fq_scales[r] = sc;
  uint32_t *orow = reinterpret_cast<uint32_t *>(args.fq_codes + static_cast<size_t>(r) * args.K);
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    float4 v[kHalf];
#pragma unroll
    for (int j = 0; j < kHalf; ++j) {
      const int i = (h * kHalf + j) * 32 + lane;
      v[j] = i < nvec ? __ldcs(xr + i) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    uint32_t redo = 0;
#pragma unroll
    for (int j = 0; j < kHalf; ++j) {
      const int i = (h * kHalf + j) * 32 + lane;
      bool tie;
      const uint32_t w = encode4_i8_fast(v[j], inv_f, tie);
      tie |= exact_row;
      if (i < nvec && !tie) orow[i] = w;
      redo |= (tie && i < nvec) ? (1u << j) : 0u;
    }
    while (redo) {
      const int j = __ffs(redo) - 1;
      redo &= redo - 1;
      const int i = (h * kHalf + j) * 32 + lane;
      orow[i] = encode4_i8_exact(__ldg(xr + i), inv);
    }
  }
  // codes and scale before the count, also for the TMA loads that read them
  fence_async_global();
  __syncwarp();
  if (lane == 0) red_release_add(args.fq_cnt + (r >> 7), 1u);
}

__device__ __forceinline__ void report_pair(int *err, volatile int *abort, uint32_t peer_abort) {
  *abort = 1;
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(peer_abort), "r"(1u) : "memory");
  if (err) atomicCAS(err, 0, ROUGE_B200_ETIMEOUT);
}

template <MmaKind KIND, int BN, bool B_MN, int OUT, bool CONV = false, bool FQ = false>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmB2, const __grid_constant__ OutMaps om,
                    const GemmArgs args) {
  using C = Cfg2<KIND, BN, B_MN, FQ>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~static_cast<uintptr_t>(1023));
  uint8_t *sA = smem;
  uint8_t *sB = smem + C::STAGES * C::A_BYTES;
  uint8_t *sSF = sB + C::STAGES * C::B_BYTES;  // block-scaled kind: [stage][SFA | SFB]
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + C::BAR_OFF);
  uint64_t *empty = full + C::STAGES;
  uint64_t *tfull = empty + C::STAGES;  // [2]
  uint64_t *tempty = tfull + 2;         // [2]
  uint64_t *mdone = tempty + 2;         // [1]
  uint64_t *ovl = mdone + 1;            // [2] overlapping accumulators: shared chunk drained
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(ovl + 2);
  volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);
  uint64_t *qbar = reinterpret_cast<uint64_t *>(smem + C::BAR_OFF + 256);  // [12] fused quantizer

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // 0: leader
  const int cluster = static_cast<int>(blockIdx.x >> 1);
  const int nclusters = static_cast<int>(gridDim.x >> 1);
  const uint32_t peer_abort = mapa_shared(smem_u32(const_cast<int *>(abort)), rank ^ 1u);

  if (threadIdx.x == 0) clock_stamp(args, 0);
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 16);
      mbar_init(&ovl[i], 8);  // the 4 warps of one column half, both CTAs
    }
    mbar_init(mdone, 1);
    if constexpr (FQ)
      for (int w = 0; w < 12; ++w) mbar_init(&qbar[w], 1);
    *abort = 0;
    mbar_init_fence();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (args.split > 1) tma_prefetch_desc(&tmB2);
    if constexpr (C::MX) {
      tma_prefetch_desc(&om.sfa);
      tma_prefetch_desc(&om.sfb);
    }
  }
  if (warp == 2) {
    tmem_alloc_pair(tmem_slot, C::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before_sync();
  cluster_sync();  // barriers of both CTAs initialised, both TMEM allocations done
  tc_fence_after_sync();
  const uint32_t tmem_base = *tmem_slot;
  // Everything above overlaps the previous kernel's tail when this launch
  // is programmatically serialised; its outputs (A, the scales) are read
  // only after this point.
  grid_dependency_wait();
  // The next programmatically serialised launch may start its own set-up
  // on SMs this grid leaves (its CTAs then wait for this grid to complete).
  grid_launch_dependents();

  if constexpr (FQ) {
    // ------------------------------------------------------------ fused quantizer
    // Every warp quantizes its rows of the first round's A blocks through a
    // 16 KB row slot of stage memory; the producer waits on named barrier 1
    // until the other eleven warps have arrived on it, before its first TMA
    // load into it. Warps 2-3 then go on with the remaining rows.
    const bool qwarp = warp == 2 || warp == 3;
    uint8_t *slot = smem + warp * C::QSLOT;
    fq_rows_first(args, slot, &qbar[warp], warp, lane);
    if (qwarp) {
      asm volatile("bar.arrive 1, 384;" ::: "memory");  // its slot is free
      for (int r = fq_claim(args, lane); r < args.M; r = fq_claim(args, lane)) fq_row_direct(args, r, lane);
    } else if (warp == 0) {
      asm volatile("bar.sync 1, 384;" ::: "memory");  // the producer: every stage slot is free
    } else {
      asm volatile("bar.arrive 1, 384;" ::: "memory");
    }
  }

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ producer
    const uint32_t full0 = mapa_shared(smem_u32(full), 0);  // leader's full[0]
    int it = 0;
    bool ok = true;
    for (int t = cluster; ok && t < args.num_tiles; t += nclusters) {
      int mb, nb, part, parts;
      unit_coords(t, args, mb, nb, part, parts);
      const int half_w = C::HALF_N / parts;                         // B rows per CTA
      const int m0 = mb * 2 * kBM + static_cast<int>(rank) * kBM;  // this CTA's A rows
      const int n0 = nb * BN + part * (BN / parts) + static_cast<int>(rank) * half_w;
      const CUtensorMap *tb = parts > 1 ? &tmB2 : &tmB;
      const uint32_t tx =
          2u * static_cast<uint32_t>(C::A_BYTES + half_w * kBKBytes + C::SFA_BYTES + C::SFB_BYTES);
      int cw = 0, ch = 0, cn = 0;
      if constexpr (CONV) conv_box(args, m0, cw, ch, cn);
      if constexpr (FQ) {  // this CTA's 128 A rows quantized (codes for the TMA loads)
        if (m0 < args.M) {
          if (!wait_count(args.fq_cnt + (m0 / kBM), static_cast<unsigned>(min(kBM, args.M - m0)),
                          abort)) {
            report_pair(args.err, abort, peer_abort);
            ok = false;
            break;
          }
          fence_async_global();
        }
      }
      for (int kb = 0; kb < args.num_k; ++kb, ++it) {
        const int s = it % C::STAGES;
        const uint32_t round = static_cast<uint32_t>(it / C::STAGES);
        if (!mbar_wait(&empty[s], (round & 1u) ^ 1u, abort)) {
          report_pair(args.err, abort, peer_abort);
          ok = false;
          break;
        }
        if (rank == 0) mbar_arrive_expect_tx(&full[s], tx);
        const uint32_t bar = full0 + static_cast<uint32_t>(s * 8);
        int kx = kb * C::BK;
        if constexpr (CONV) {
          int c0, kr, kc;
          conv_kblock(args, kb, C::BK, c0, kr, kc, kx);
          tma_load_im2col_4d_pair(sA + s * C::A_BYTES, &tmA, bar, c0, cw, ch, cn,
                                  static_cast<uint16_t>(kc), static_cast<uint16_t>(kr));
        } else {
          tma_load_2d_pair(sA + s * C::A_BYTES, &tmA, bar, kx, m0);
        }
        if constexpr (C::MX) {  // scale atoms: A rows m0.., all BN B rows of the tile
          uint8_t *sf = sSF + s * C::SF_STAGE;
          constexpr int kRows = 4 * C::ATOMS_K;  // 128-byte rows of this stage's atoms
          tma_load_2d_pair(sf, &om.sfa, bar, 0, ((m0 / kBM) * args.sf_kblocks + kb) * kRows);
#pragma unroll
          for (int j = 0; j < BN / 128; ++j)
            tma_load_2d_pair(sf + C::SFA_BYTES + j * C::ATOMS_K * 512, &om.sfb, bar, 0,
                             ((nb * BN / 128 + j) * args.sf_kblocks + kb) * kRows);
        }
        if constexpr (!B_MN) {
          tma_load_2d_pair(sB + s * C::B_BYTES, tb, bar, kx,
                           n0 + (args.item_m ? (m0 / args.item_m) * args.N : 0));
        } else {  // (no split units with MN-major B)
#pragma unroll
          for (int j = 0; j < C::B_CHUNKS; ++j)
            tma_load_2d_pair(sB + s * C::B_BYTES + j * C::B_CHUNK_BYTES, &tmB, bar,
                             n0 + j * (kBKBytes / C::ESIZE), kb * C::BK);
        }
      }
    }
    // Wait for the leader's releases of the last stages, so that no commit
    // from the leader's MMA is still to arrive on this CTA's barriers when
    // the cluster exits (on the abort path, so that the leader's full
    // barriers have seen the last loads land: best effort, bounded).
    const volatile int never = 0;
    for (int j = (it > C::STAGES ? it - C::STAGES : 0); j < it; ++j) {
      if (ok) {
        if (!mbar_wait(&empty[j % C::STAGES], static_cast<uint32_t>(j / C::STAGES) & 1u, abort)) {
          report_pair(args.err, abort, peer_abort);
          ok = false;
        }
      } else if (rank == 0) {
        mbar_wait(&full[j % C::STAGES], static_cast<uint32_t>(j / C::STAGES) & 1u, &never);
      }
    }
  } else if (warp == 1 && lane == 0 && rank == 0) {
    // ------------------------------------------------------------ MMA issuer (leader)
    constexpr uint32_t c_fmt = KIND == MmaKind::I8 ? 2u : 1u;
    constexpr uint32_t ab_fmt = KIND == MmaKind::I8 ? 1u : (KIND == MmaKind::TF32 ? 2u : 0u);
    const uint32_t ab = (KIND == MmaKind::F16 && args.bf16) ? 1u : ab_fmt;
    // block-scaled: E8M0 scales (format 1) for MXF8, UE4M3 (0) for NVF4
    constexpr uint32_t sf_fmt = C::NV ? 0u : 1u;  // (MXF4: E8M0)
    const uint32_t idesc_full =
        C::MX ? make_idesc_mx(static_cast<uint32_t>(args.mx_fmt_a), static_cast<uint32_t>(args.mx_fmt_b),
                              2 * kBM, BN, sf_fmt, 0u, 0u)
              : make_idesc(c_fmt, ab, ab, 0u, B_MN ? 1u : 0u, 2 * kBM, BN);
    const uint32_t idesc_part =
        C::MX ? make_idesc_mx(static_cast<uint32_t>(args.mx_fmt_a), static_cast<uint32_t>(args.mx_fmt_b),
                              2 * kBM, BN / (args.split > 1 ? args.split : 1), sf_fmt, 0u, 0u)
              : make_idesc(c_fmt, ab, ab, 0u, B_MN ? 1u : 0u, 2 * kBM,
                           BN / (args.split > 1 ? args.split : 1));
    const uint32_t empty_peer = mapa_shared(smem_u32(empty), 1);
    const uint32_t tfull_peer = mapa_shared(smem_u32(tfull), 1);
    int it = 0, local = 0;
    bool ok = true;
    bool issued = false;
    for (int t = cluster; ok && t < args.num_tiles; t += nclusters, ++local) {
      const int slot = local & 1;
      const uint32_t use = static_cast<uint32_t>(local >> 1);
      if (!mbar_wait(&tempty[slot], (use & 1u) ^ 1u, abort)) {
        report_pair(args.err, abort, peer_abort);
        ok = false;
        break;
      }
      if constexpr (C::OVERLAP) {
        // the previous tile's epilogue has drained the chunk both buffers share
        if (local > 0 &&
            !mbar_wait(&ovl[slot ^ 1], static_cast<uint32_t>((local - 1) >> 1) & 1u, abort)) {
          report_pair(args.err, abort, peer_abort);
          ok = false;
          break;
        }
      }
      tc_fence_after_sync();
      const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(slot * C::ACC1_COL);
      const uint32_t idesc = t >= args.split_from ? idesc_part : idesc_full;
      // block-scaled split unit: its B rows' scale words start 4 columns per
      // 128 rows into the tile's SFB
      uint32_t sfb_unit = 0;
      if constexpr (C::MX) {
        int mb_, nb_, part_, parts_;
        unit_coords(t, args, mb_, nb_, part_, parts_);
        sfb_unit = static_cast<uint32_t>(part_ * (BN / parts_) / 128) * 4u;
      }
      for (int kb = 0; kb < args.num_k; ++kb, ++it) {
        const int s = it % C::STAGES;
        const uint32_t round = static_cast<uint32_t>(it / C::STAGES);
        if (!mbar_wait(&full[s], round & 1u, abort)) {
          report_pair(args.err, abort, peer_abort);
          ok = false;
          break;
        }
        tc_fence_after_sync();
        const uint32_t a0 = smem_u32(sA + s * C::A_BYTES);
        const uint32_t b0 = smem_u32(sB + s * C::B_BYTES);
        if constexpr (C::MX) {
          // This stage's scale atoms into TMEM (after the previous k-block's
          // MMAs, which read the same columns: same-thread order). MXF8: one
          // MMA per 32 K reading byte k of every scale word (SFA at t_sf,
          // SFB at t_sf + 4); NVF4: one MMA per 64 K reading whole words of
          // its own atoms (SFA k at t_sf + 4k, SFB k at t_sf + 16 + 8k).
          const uint32_t sf0 = smem_u32(sSF + s * C::SF_STAGE);
          const uint32_t t_sf =
              tmem_base + static_cast<uint32_t>(C::SF_COL + (it % C::SF_BUFS) * C::SF_SET);
          constexpr uint32_t kSfbCol = 4u * C::ATOMS_K;  // SFB after the SFA atoms
#pragma unroll
          for (int a = 0; a < C::ATOMS_K; ++a)
            tc_cp_32x128b_x4_pair(t_sf + 4u * a, smem_desc_noswizzle(sf0 + 512 * a, 128, 128));
#pragma unroll
          for (int j = 0; j < BN / 128; ++j)
#pragma unroll
            for (int a = 0; a < C::ATOMS_K; ++a)
              tc_cp_32x128b_x4_pair(
                  t_sf + kSfbCol + static_cast<uint32_t>(a * (BN / 32) + 4 * j),
                  smem_desc_noswizzle(sf0 + C::SFA_BYTES + 512 * (j * C::ATOMS_K + a), 128, 128));
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint32_t kk = static_cast<uint32_t>(k);
            const uint64_t adesc = smem_desc_sw128(a0 + k * 32, 16, 1024);
            const uint64_t bdesc = smem_desc_sw128(b0 + k * 32, 16, 1024);
            const uint32_t acc = (kb | k) != 0 ? 1u : 0u;
            if constexpr (C::NV) {
              umma_nvf4_pair(d_tmem, adesc, bdesc, idesc, t_sf + 4u * kk,
                             t_sf + kSfbCol + kk * (BN / 32) + sfb_unit, acc);
            } else if constexpr (C::F4) {  // atom k / 2, byte pair 2 (k % 2)
              const uint32_t id = (kk & 1u) * 2u;
              umma_mxf4_pair(d_tmem, adesc, bdesc, idesc | (id << 29) | (id << 4),
                             (t_sf + 4u * (kk >> 1)) | (id << 30),
                             (t_sf + kSfbCol + (kk >> 1) * (BN / 32) + sfb_unit) | (id << 30), acc);
            } else
              umma_mx_pair(d_tmem, adesc, bdesc, idesc | (kk << 29) | (kk << 4), t_sf | (kk << 30),
                           (t_sf + kSfbCol + sfb_unit) | (kk << 30), acc);
          }
        } else {
#pragma unroll
          for (int k = 0; k < C::BK / C::UMMA_K; ++k) {
            const uint64_t adesc = smem_desc_sw128(a0 + k * 32, 16, 1024);
            const uint64_t bdesc =
                B_MN ? smem_desc_sw128(b0 + k * C::UMMA_K * kBKBytes, C::B_CHUNK_BYTES, 1024)
                     : smem_desc_sw128(b0 + k * 32, 16, 1024);
            umma_pair<KIND>(d_tmem, adesc, bdesc, idesc, (kb | k) != 0 ? 1u : 0u);
          }
        }
        issued = true;
        tc_commit_pair(smem_u32(&empty[s]));
        tc_commit_pair(empty_peer + static_cast<uint32_t>(s * 8));
      }
      if (!ok) break;
      tc_commit_pair(smem_u32(&tfull[slot]));
      tc_commit_pair(tfull_peer + static_cast<uint32_t>(slot * 8));
    }
    if (!ok && issued) {
      const volatile int never = 0;
      tc_commit_pair(smem_u32(mdone));
      mbar_wait(mdone, 0u, &never);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int quarter = warp & 3;
    const int half = (warp - 4) >> 2;
    uint8_t *stage = smem + C::STAGES * C::STAGE_BYTES + (warp - 4) * C::EPI_BUFS * kStageBytes;
    const uint32_t tempty0 = mapa_shared(smem_u32(tempty), 0);  // leader's tempty[0]
    const uint32_t ovl0 = mapa_shared(smem_u32(ovl), 0);        // leader's ovl[0]
    int local = 0, seq = 0;
    float sab = 1.0f;
    if constexpr (KIND != MmaKind::I8) {
      if (args.scale_a && args.scale_b) sab = x86_mul(__ldg(args.scale_a), __ldg(args.scale_b));
      if (args.blas) sab = args.alpha;
    }
    bool fq_more = FQ;  // rows of A left to claim
    for (int t = cluster; t < args.num_tiles; t += nclusters, ++local) {
      int mb, nb, part, parts;
      unit_coords(t, args, mb, nb, part, parts);
      const int slot = local & 1;
      const uint32_t use = static_cast<uint32_t>(local >> 1);
      if constexpr (FQ) {
        // code rows of A while this tile's accumulator is not ready (a row
        // takes a few microseconds; the other accumulator buffer keeps the
        // MMA busy meanwhile)
        while (fq_more && !__any_sync(0xffffffffu, mbar_test_wait(&tfull[slot], use & 1u))) {
          const int r = fq_claim(args, lane);
          if (r >= args.M) {
            fq_more = false;
            break;
          }
          fq_row_direct(args, r, lane);
        }
      }
      if (!mbar_wait(&tfull[slot], use & 1u, abort)) {
        report_pair(args.err, abort, peer_abort);
        break;
      }
      tc_fence_after_sync();
      if constexpr (FQ) {  // the rows' scales (complete: the tile's codes were)
        const int m0 = mb * 2 * kBM + static_cast<int>(rank) * kBM;
        if (m0 < args.M &&
            !wait_count(args.fq_cnt + (m0 / kBM), static_cast<unsigned>(min(kBM, args.M - m0)), abort)) {
          report_pair(args.err, abort, peer_abort);
          break;
        }
      }
      epilogue_tile<KIND, OUT, C::EPI_BUFS>(
          args, tmem_base + static_cast<uint32_t>(slot * C::ACC1_COL),
          mb * 2 * kBM + static_cast<int>(rank) * kBM, nb * BN + part * (BN / parts), BN / parts,
          quarter, half, sab, stage, seq, &om, lane,
          C::OVERLAP ? ovl0 + static_cast<uint32_t>(slot * 8) : 0u,
          // buffer 0: the shared columns are its chunk ACC1_COL/32 (held
          // only by full-width tiles); buffer 1: its first chunk
          slot == 0 ? 1 : 0,
          slot == 0 ? (BN / parts > C::ACC1_COL ? C::ACC1_COL / 32 : -1) : 0, C::OVL_CHUNKS);
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty0 + static_cast<uint32_t>(slot * 8));
    }
    if (args.use_tma_store && lane == 0) bulk_wait_all();
    // Broadcast stores reach other GPUs: order them before anything this
    // thread's kernel completion releases (the cross-rank barrier after it).
    if (args.bcast || args.npeers) asm volatile("fence.acq_rel.sys;" ::: "memory");
  }

  tc_fence_before_sync();
  cluster_sync();  // all MMAs into both TMEMs done, no remote arrivals pending
  if (warp == 2) {
    tc_fence_after_sync();
    tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
  }
  if constexpr (FQ) {
    // The last CTA to finish zeroes the block counts for the next launch
    // (every other CTA is past its last use of them).
    if (threadIdx.x == 0) {
      const int nblk = (args.M + kBM - 1) / kBM;
      if (atom_add_acq_rel(args.fq_cnt + nblk, 1u) == gridDim.x - 1u) {
        for (int b = 0; b <= nblk + 1; ++b) args.fq_cnt[b] = 0u;
      }
    }
  }
  if (threadIdx.x == 0) clock_stamp(args, 2);
}

// The clock probe of rouge_b200_set_clock_probe: stamp buffer, its CTA
// capacity and the device it lives on (launches on other devices skip it).
std::atomic<unsigned long long *> g_clock_stamps{nullptr};
std::atomic<int> g_clock_ctas{0};
std::atomic<int> g_clock_dev{-1};

// Builds the output map and launches one GEMM / convolution.
// make_b(box_rows, map) encodes the B operand's tensor map with boxes of
// `box_rows` rows (K-major B) and returns a status.
template <MmaKind KIND, int BN, bool B_MN, int OUT, bool CONV, bool PAIR, bool FQ = false, class MakeB>
int launch_tiles(const CUtensorMap &ta, MakeB make_b, GemmArgs args, cudaStream_t st) {
  int s = ROUGE_B200_OK;
  if (unsigned long long *stamps = g_clock_stamps.load()) {
    if (g_clock_dev.load() == current_device()) {
      args.clk = stamps;
      args.clk_n = g_clock_ctas.load();
    }
  }
  CUtensorMap tb;
  s = make_b(PAIR ? BN / 2 : BN, &tb);
  if (s != ROUGE_B200_OK) return s;
  // Output map for the epilogue's TMA stores: 32 x 32 boxes, swizzle
  // matching the staging layout (128 B rows for 4-byte, 64 B for bf16).
  // Broadcast through peer pointers: one map per rank over that rank's copy
  // of this GEMM's column block (clipping at the block's edges).
  OutMaps tc;
  std::memset(&tc, 0, sizeof(tc));
  const bool b16 = OUT == ROUGE_B200_OUT_BF16;
  const CUtensorMapDataType odt = b16 ? CU_TENSOR_MAP_DATA_TYPE_UINT16 : CU_TENSOR_MAP_DATA_TYPE_UINT32;
  const CUtensorMapSwizzle osw = b16 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B;
  const int oes = b16 ? 2 : 4;
  if (args.npeers) {
    // bf16: whole 64-column lines (128-byte rows) per box, see peer_flush
    for (int r = 0; r < args.npeers; ++r) {
      s = make_tmap_2d(&tc.m[r], static_cast<uint8_t *>(args.peers[r]) +
                                     static_cast<size_t>(args.col_off) * oes,
                       odt, args.N, args.M, static_cast<uint64_t>(args.bld) * oes, b16 ? 64 : 32,
                       32, CU_TENSOR_MAP_SWIZZLE_128B);
      if (s != ROUGE_B200_OK) return s;
    }
    tc.n = args.npeers;
    args.use_tma_store = 1;
  } else if (args.use_tma_store) {
    s = make_tmap_2d(&tc.m[0], args.C, odt, args.N, args.M,
                     static_cast<uint64_t>(args.ldc) * oes, 32, 32, osw);
    if (s != ROUGE_B200_OK) return s;
    tc.n = 1;
  }
  if constexpr (KIND == MmaKind::MXF8 || KIND == MmaKind::NVF4 || KIND == MmaKind::MXF4) {
    // scale atoms as 128-byte rows, 4 rows per atom, one stage's atoms
    // (1 for MXF8, 2 for MXF4, 4 for NVF4) per box, no swizzle
    const uint32_t box = KIND == MmaKind::NVF4 ? 16u : (KIND == MmaKind::MXF4 ? 8u : 4u);
    const uint64_t rows_a = static_cast<uint64_t>((args.M + 127) / 128) * args.sf_kblocks * box;
    const uint64_t rows_b = static_cast<uint64_t>((args.N + 127) / 128) * args.sf_kblocks * box;
    s = make_tmap_2d(&tc.sfa, args.scales_a, CU_TENSOR_MAP_DATA_TYPE_UINT8, 128, rows_a, 128, 128,
                     box, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (s == ROUGE_B200_OK)
      s = make_tmap_2d(&tc.sfb, args.scales_b, CU_TENSOR_MAP_DATA_TYPE_UINT8, 128, rows_b, 128, 128,
                       box, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (s != ROUGE_B200_OK) return s;
  }

  const unsigned long long bit = 1ull << (current_device() & 63);
  const int sms = current_sm_count();
  if constexpr (!PAIR) {
    using C = Cfg<KIND, BN, B_MN>;
    auto kern = gemm_tc_kernel<KIND, BN, B_MN, OUT, CONV>;
    // The shared-memory opt-in is a per-device function attribute.
    static std::atomic<unsigned long long> attr_done{0};
    if (!(attr_done.load() & bit)) {
      s = cuda_status(
          cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
      if (s != ROUGE_B200_OK) return s;
      attr_done.fetch_or(bit);
    }
    const int grid = args.num_tiles < sms ? args.num_tiles : sms;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid, 1, 1);
    cfg.blockDim = dim3(kGemmThreads, 1, 1);
    cfg.dynamicSmemBytes = C::SMEM;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cuda_status(cudaLaunchKernelEx(&cfg, kern, ta, tb, tc, args));
  } else {
    using C = Cfg2<KIND, BN, B_MN, FQ>;
    auto kern = gemm_tc2_kernel<KIND, BN, B_MN, OUT, CONV, FQ>;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim = dim3(kGemmThreads, 1, 1);
    cfg.dynamicSmemBytes = C::SMEM;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    // Per device: the shared-memory opt-in, then how many 2-CTA clusters of
    // this kernel fit on the GPU at once (SM pairs of one TPC).
    static std::atomic<unsigned long long> attr_done{0};
    static std::atomic<int> max_clusters[64];
    const int dev = current_device() & 63;
    if (!(attr_done.load() & bit)) {
      s = cuda_status(
          cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
      if (s != ROUGE_B200_OK) return s;
      cfg.gridDim = dim3(2, 1, 1);
      int n = 0;
      s = cuda_status(cudaOccupancyMaxActiveClusters(&n, kern, &cfg));
      if (s != ROUGE_B200_OK) return s;
      if (n < 1) return set_status(ROUGE_B200_EUNSUPPORTED);
      max_clusters[dev].store(n);
      attr_done.fetch_or(bit);
    }
    int clusters = max_clusters[dev].load();
    if (clusters > sms / 2) clusters = sms / 2 > 0 ? sms / 2 : 1;
    // Last partial round: cut its tiles N-wise into 2 or 4 units when that
    // many units still fit in one round (K-major B only).
    const int tiles = args.num_tiles;
    const int rem = tiles % clusters;
    args.split_from = tiles;
    args.split = 1;
#ifndef RB200_MAX_SPLIT  // largest N-split of the last round (tuning builds)
#define RB200_MAX_SPLIT 2
#endif
    // (block-scaled: only halves, whose B rows are one whole scale atom)
    const int max_split =
        KIND == MmaKind::MXF8 || KIND == MmaKind::NVF4 || KIND == MmaKind::MXF4 ? 2 : RB200_MAX_SPLIT;
    if (!B_MN && rem) {
      for (int f = max_split; f >= 2; f /= 2) {
        if (rem * f <= clusters) {
          args.split = f;
          break;
        }
      }
    }
    CUtensorMap tb2 = tb;
    if (args.split > 1) {
      args.split_from = tiles - rem;
      args.num_tiles = args.split_from + rem * args.split;
      s = make_b(BN / 2 / args.split, &tb2);
      if (s != ROUGE_B200_OK) return s;
    }
    if (clusters > args.num_tiles) clusters = args.num_tiles;
    if constexpr (FQ) {
      // rows of the A blocks the first RB200_FQ_ROUNDS rounds of units need
      // (units walk N first, so a round's last unit has its largest m-block)
#ifndef RB200_FQ_ROUNDS  // rounds quantized before the tiles start (tuning builds)
#define RB200_FQ_ROUNDS 1
#endif
      const int u = (args.num_tiles < RB200_FQ_ROUNDS * clusters ? args.num_tiles
                                                                  : RB200_FQ_ROUNDS * clusters) - 1;
      const int t = u >= args.split_from ? args.split_from + (u - args.split_from) / args.split : u;
      const long long rows = RB200_FQ_ROUNDS > 0 ? static_cast<long long>(t / args.num_n + 1) * 2 * kBM : 0;
      args.fq_rows0 = rows < args.M ? static_cast<int>(rows) : args.M;
    }
    cfg.gridDim = dim3(2 * clusters, 1, 1);
    return cuda_status(cudaLaunchKernelEx(&cfg, kern, ta, tb, tb2, tc, args));
  }
}

template <MmaKind KIND, int BN, bool B_MN, int OUT, bool PAIR>
int launch_gemm_impl(const void *A, long long lda, const void *B, long long ldb, GemmArgs args,
                     cudaStream_t st) {
  using C = Cfg<KIND, BN, B_MN>;
  const CUtensorMapDataType dt = C::ESIZE == 4   ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : C::ESIZE == 2 ? CU_TENSOR_MAP_DATA_TYPE_UINT16
                                                 : CU_TENSOR_MAP_DATA_TYPE_UINT8;
  CUtensorMap ta;
  int s = make_tmap_2d(&ta, A, dt, args.K, args.M, static_cast<uint64_t>(lda) * C::ESIZE, C::BK,
                       kBM);
  if (s != ROUGE_B200_OK) return s;
  auto make_b = [&](int box_rows, CUtensorMap *tb) {
    if (!B_MN)  // K-major: boxes of box_rows rows of B (every item's rows when batched)
      return make_tmap_2d(tb, B, dt, args.K,
                          static_cast<uint64_t>(args.N) * (args.item_m ? args.M / args.item_m : 1),
                          static_cast<uint64_t>(ldb) * C::ESIZE, C::BK, box_rows);
    return make_tmap_2d(tb, B, dt, args.N, args.K, static_cast<uint64_t>(ldb) * C::ESIZE,
                        kBKBytes / C::ESIZE, C::BK);
  };
  return launch_tiles<KIND, BN, B_MN, OUT, false, PAIR>(ta, make_b, args, st);
}

template <MmaKind KIND, int BN, bool B_MN, bool PAIR>
int launch_out(const void *A, long long lda, const void *B, long long ldb, GemmArgs args,
               int out_type, cudaStream_t st) {
  switch (out_type) {
    case ROUGE_B200_OUT_F32:
      return launch_gemm_impl<KIND, BN, B_MN, ROUGE_B200_OUT_F32, PAIR>(A, lda, B, ldb, args, st);
    case ROUGE_B200_OUT_BF16:
      return launch_gemm_impl<KIND, BN, B_MN, ROUGE_B200_OUT_BF16, PAIR>(A, lda, B, ldb, args, st);
    default:
      if constexpr (KIND == MmaKind::I8)
        return launch_gemm_impl<KIND, BN, B_MN, ROUGE_B200_OUT_I32, PAIR>(A, lda, B, ldb, args,
                                                                          st);
      return set_status(ROUGE_B200_EINVAL);
  }
}

// Tile shape chooser. A wave of 256 x 256 CTA-pair tiles whenever the
// 128 x 256 tiles fill every SM at least once (same tile count per SM, half
// the operand reads per output); otherwise 128 x 128 single-CTA tiles, which
// spread a small problem over more SMs (128 x 64 or 128 x 32 when even those
// leave most SMs idle, launch_kind). rouge_b200_set_tile_mode overrides.
std::atomic<int> g_tile_mode{ROUGE_B200_TILES_AUTO};

bool use_pair_tiles(int M, int N) {
  const int mode = g_tile_mode.load();
  if (mode != ROUGE_B200_TILES_AUTO) return mode == ROUGE_B200_TILES_PAIR;
  const long long tiles256 = static_cast<long long>((M + kBM - 1) / kBM) * ((N + 255) / 256);
  return tiles256 >= current_sm_count();
}

template <MmaKind KIND>
int launch_kind(const void *A, long long lda, const void *B, long long ldb, int b_layout,
                GemmArgs args, int out_type, cudaStream_t st) {
  const bool pair = args.tile_hint != kTileHintAuto ? args.tile_hint == kTileHintPair
                                                    : use_pair_tiles(args.M, args.N);
  // Single-CTA tiles: BN = 256 unless that leaves most SMs idle; then 128.
  const long long tiles256 =
      static_cast<long long>((args.M + kBM - 1) / kBM) * ((args.N + 255) / 256);
#ifdef RB200_FORCE_BN  // compile-time tile override for tuning builds
  const int bn = pair ? 256 : RB200_FORCE_BN;
  (void)tiles256;
#else
  const int bn = pair ? 256
                 : args.tile_hint == kTileHintSingle128 ? 128
                 : args.tile_hint == kTileHintSingle256 ? 256
                 : (tiles256 >= current_sm_count() ? 256 : 128);
#endif
  const int bm = pair ? 2 * kBM : kBM;
  args.num_m = (args.M + bm - 1) / bm;
  args.num_n = (args.N + bn - 1) / bn;
  const int esize = KIND == MmaKind::TF32 ? 4 : (KIND == MmaKind::F16 ? 2 : 1);
  const int bk = kBKBytes / esize;
  args.num_k = (args.K + bk - 1) / bk;
  args.num_tiles = args.num_m * args.num_n;
  const bool mn = b_layout == ROUGE_B200_B_KN;
  if (pair)
    return mn ? launch_out<KIND, 256, true, true>(A, lda, B, ldb, args, out_type, st)
              : launch_out<KIND, 256, false, true>(A, lda, B, ldb, args, out_type, st);
  if (bn == 256)
    return mn ? launch_out<KIND, 256, true, false>(A, lda, B, ldb, args, out_type, st)
              : launch_out<KIND, 256, false, false>(A, lda, B, ldb, args, out_type, st);
  // Few 128 x 128 tiles (at most one per two SMs): 128 x 64 or 128 x 32
  // tiles (K-major B, plain output) put two or four times as many SMs on
  // the operand feed, shrink each CTA's epilogue and keep a K of up to 8
  // k-blocks in flight at once in the stage ring.
  if (!mn && args.tile_hint == kTileHintAuto && !args.bcast && !args.npeers &&
      2 * args.num_tiles <= current_sm_count()) {
    const bool n32 = 4 * args.num_tiles <= current_sm_count();
    args.num_n = (args.N + (n32 ? 31 : 63)) / (n32 ? 32 : 64);
    args.num_tiles = args.num_m * args.num_n;
    return n32 ? launch_out<KIND, 32, false, false>(A, lda, B, ldb, args, out_type, st)
               : launch_out<KIND, 64, false, false>(A, lda, B, ldb, args, out_type, st);
  }
  return mn ? launch_out<KIND, 128, true, false>(A, lda, B, ldb, args, out_type, st)
            : launch_out<KIND, 128, false, false>(A, lda, B, ldb, args, out_type, st);
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

template <MmaKind KIND, int BN, bool PAIR, int OUT>
int launch_conv_bn(const CUtensorMap &ta, const void *Wt, GemmArgs g, cudaStream_t st) {
  using C = Cfg<KIND, BN, false>;
  auto make_b = [&](int box_rows, CUtensorMap *tb) {
    return make_tmap_2d(tb, Wt,
                        C::ESIZE == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                      : CU_TENSOR_MAP_DATA_TYPE_UINT16,
                        g.K, g.N, static_cast<uint64_t>(g.K) * C::ESIZE, C::BK, box_rows);
  };
  return launch_tiles<KIND, BN, false, OUT, true, PAIR>(ta, make_b, g, st);
}

}  // namespace

// Implicit-GEMM convolution, NHWC in, f32 NHWC out (+ bias): f16/bf16
// inputs (kind::f16, 64 channels per k-block) or f32 inputs read as tf32
// (kind::tf32, 32 channels per k-block).
// GEMM view: M = N*OH*OW output pixels, N = Cout, K = KH*KW*Cin in
// (kr, kc, c) order, so the weights [Cout][KH][KW][Cin] are the K-major B
// operand as stored. The A tile of k-block (tap, c0) is one im2col TMA load:
// 128 consecutive output pixels (crossing rows and images) x BK channels of
// filter tap (kr, kc), zeros in the padding. Y has row pitch ldy >= Cout
// and element type out_type: f32, or 16-bit (kind::f16 only) holding bf16
// or, with f16out, IEEE half. blas != 0: Y = alpha * acc + beta * Y (no
// bias), the old Y read only when beta != 0.
template <MmaKind KIND>
int launch_conv(int N, int H, int W, int Cin, int Cout, int KH, int KW, int stride, int pad,
                const void *X, const void *Wt, const float *bias, void *Y, long long ldy,
                int is_bf16, int out_type, int f16out, int blas, float alpha, float beta,
                cudaStream_t st) {
  using C0 = Cfg<KIND, 128, false>;
  const int OH = (H + 2 * pad - KH) / stride + 1, OW = (W + 2 * pad - KW) / stride + 1;
  GemmArgs g{};
  g.M = N * OH * OW;
  g.N = Cout;
  g.K = KH * KW * Cin;
  g.C = Y;
  g.ldc = ldy;
  g.bf16 = is_bf16 ? 1 : 0;
  g.bias = bias;
  g.vec16 = (reinterpret_cast<uintptr_t>(bias) & 15u) == 0;
  g.use_tma_store = vec_ok(Y, ldy, out_type);
  g.f16out = f16out;
  g.blas = blas;
  g.alpha = alpha;
  g.beta = beta;
  g.err = device_error_word();
  g.conv_cblocks = Cin / C0::BK;
  g.conv_kw = KW;
  g.conv_oh = OH;
  g.conv_ow = OW;
  g.conv_stride = stride;
  g.conv_pad = pad;
  g.conv_cin = Cin;
  CUtensorMap ta;
  int s = make_tmap_im2col_nhwc(&ta, X,
                                C0::ESIZE == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                               : CU_TENSOR_MAP_DATA_TYPE_UINT16,
                                C0::ESIZE, N, H, W, Cin, -pad, -pad, pad - (KW - 1), pad - (KH - 1),
                                C0::BK, kBM, stride, stride);
  if (s != ROUGE_B200_OK) return s;
  const int sms = current_sm_count();
  const long long tiles256 = static_cast<long long>((g.M + kBM - 1) / kBM) * ((Cout + 255) / 256);
  const bool pair = g_tile_mode.load() == ROUGE_B200_TILES_AUTO
                        ? (Cout > 128 && tiles256 >= sms)
                        : g_tile_mode.load() == ROUGE_B200_TILES_PAIR;
  const int bn = (pair || (Cout > 128 && tiles256 >= sms)) ? 256 : 128;
  const int bm = pair ? 2 * kBM : kBM;
  g.num_m = (g.M + bm - 1) / bm;
  g.num_n = (Cout + bn - 1) / bn;
  g.num_k = KH * KW * g.conv_cblocks;
  g.num_tiles = g.num_m * g.num_n;
  if constexpr (KIND == MmaKind::F16) {
    if (out_type == ROUGE_B200_OUT_BF16) {
      if (pair) return launch_conv_bn<KIND, 256, true, ROUGE_B200_OUT_BF16>(ta, Wt, g, st);
      return bn == 256 ? launch_conv_bn<KIND, 256, false, ROUGE_B200_OUT_BF16>(ta, Wt, g, st)
                       : launch_conv_bn<KIND, 128, false, ROUGE_B200_OUT_BF16>(ta, Wt, g, st);
    }
  }
  if (out_type != ROUGE_B200_OUT_F32) return set_status(ROUGE_B200_EUNSUPPORTED);
  if (pair) return launch_conv_bn<KIND, 256, true, ROUGE_B200_OUT_F32>(ta, Wt, g, st);
  return bn == 256 ? launch_conv_bn<KIND, 256, false, ROUGE_B200_OUT_F32>(ta, Wt, g, st)
                   : launch_conv_bn<KIND, 128, false, ROUGE_B200_OUT_F32>(ta, Wt, g, st);
}

int launch_conv_f16(int N, int H, int W, int Cin, int Cout, int KH, int KW, int stride, int pad,
                    const uint16_t *X, const uint16_t *Wt, const float *bias, float *Y,
                    int is_bf16, cudaStream_t st) {
  return launch_conv<MmaKind::F16>(N, H, W, Cin, Cout, KH, KW, stride, pad, X, Wt, bias, Y, Cout,
                                   is_bf16, ROUGE_B200_OUT_F32, 0, 0, 1.0f, 0.0f, st);
}

// f32 NHWC convolution with tf32 operands (Cin a multiple of 32, inputs of
// at least 128 KB, 16-byte aligned X and Wt).
int launch_conv_tf32(int N, int H, int W, int Cin, int Cout, int KH, int KW, int stride, int pad,
                     const float *X, const float *Wt, const float *bias, float *Y, long long ldy,
                     cudaStream_t st) {
  return launch_conv<MmaKind::TF32>(N, H, W, Cin, Cout, KH, KW, stride, pad, X, Wt, bias, Y, ldy,
                                    0, ROUGE_B200_OUT_F32, 0, 0, 1.0f, 0.0f, st);
}

// The cuDNN-forward form: Y (row pitch ldy, element type y_type: T_F32,
// T_F16 or T_BF16) = alpha * conv(X, Wt) + beta * Y. ab_type T_F16 / T_BF16
// (kind::f16, Cin % 64 == 0) or T_F32 (kind::tf32, Cin % 32 == 0; the
// caller splits operands for f32 accuracy). Checked by the caller.
int launch_conv_blas(int ab_type, int N, int H, int W, int Cin, int Cout, int KH, int KW,
                     int stride, int pad, const void *X, const void *Wt, float alpha, float beta,
                     void *Y, long long ldy, int y_type, cudaStream_t st) {
  const int out = y_type == ROUGE_B200_T_F32 ? ROUGE_B200_OUT_F32 : ROUGE_B200_OUT_BF16;
  const int f16out = y_type == ROUGE_B200_T_F16 ? 1 : 0;
  if (ab_type == ROUGE_B200_T_F32)
    return launch_conv<MmaKind::TF32>(N, H, W, Cin, Cout, KH, KW, stride, pad, X, Wt, nullptr, Y,
                                      ldy, 0, out, f16out, 1, alpha, beta, st);
  return launch_conv<MmaKind::F16>(N, H, W, Cin, Cout, KH, KW, stride, pad, X, Wt, nullptr, Y, ldy,
                                   ab_type == ROUGE_B200_T_BF16 ? 1 : 0, out, f16out, 1, alpha, beta,
                                   st);
}

int launch_gemm_i8(int M, int N, int K, const int8_t *A, long long lda, const int8_t *B,
                   long long ldb, int b_layout, const float *sa, int a_rows, const float *sb,
                   int b_cols, void *Cp, long long ldc, int out_type, cudaStream_t st) {
  GemmArgs g{};
  g.M = M; g.N = N; g.K = K;
  g.C = Cp; g.ldc = ldc;
  g.scales_a = sa; g.scales_b = sb; g.a_rows = a_rows; g.b_cols = b_cols;
  g.use_tma_store = vec_ok(Cp, ldc, out_type);
  g.vec16 = (reinterpret_cast<uintptr_t>(sb) & 15u) == 0;
  g.err = device_error_word();
  return launch_kind<MmaKind::I8>(A, lda, B, ldb, b_layout, g, out_type, st);
}

int launch_quant_i8_rows(const float *x, int rows, int cols, float *scales, int8_t *out,
                         cudaStream_t st);

// The W8A8 linear step: per-row quantization of X (codes Aq, scales sa)
// and C = dequant(Aq . Wq^T). One launch of the CTA-pair int8 kernel with
// the quantizer fused (see GemmArgs::fq_x) when K <= 4096 (a row fits a
// 16 KB slot) and the problem takes CTA-pair tiles; otherwise the row
// quantizer, then the GEMM.
int launch_w8a8_linear(int M, int N, int K, const float *X, const int8_t *Wq, const float *sw,
                       int8_t *Aq, float *sa, void *Cp, long long ldc, int out_type, unsigned *ws,
                       cudaStream_t st) {
  const bool fuse = K <= 4096 && (reinterpret_cast<uintptr_t>(X) & 15u) == 0 && use_pair_tiles(M, N);
  if (!fuse) {
    int s = launch_quant_i8_rows(X, M, K, sa, Aq, st);
    if (s != ROUGE_B200_OK) return s;
    return launch_gemm_i8(M, N, K, Aq, K, Wq, K, ROUGE_B200_B_NK, sa, 1, sw, 1, Cp, ldc, out_type,
                          st);
  }
  GemmArgs g{};
  g.M = M; g.N = N; g.K = K;
  g.C = Cp; g.ldc = ldc;
  g.scales_a = sa; g.scales_b = sw; g.a_rows = 1; g.b_cols = 1;
  g.use_tma_store = vec_ok(Cp, ldc, out_type);
  g.vec16 = (reinterpret_cast<uintptr_t>(sw) & 15u) == 0;
  g.err = device_error_word();
  g.fq_x = X;
  g.fq_codes = Aq;
  g.fq_scales = sa;
  g.fq_cnt = ws;
  g.n_fast = 1;
  g.num_m = (M + 2 * kBM - 1) / (2 * kBM);
  g.num_n = (N + 255) / 256;
  g.num_k = (K + kBKBytes - 1) / kBKBytes;
  g.num_tiles = g.num_m * g.num_n;
  CUtensorMap ta;
  int s = make_tmap_2d(&ta, Aq, CU_TENSOR_MAP_DATA_TYPE_UINT8, K, M, static_cast<uint64_t>(K),
                       kBKBytes, kBM);
  if (s != ROUGE_B200_OK) return s;
  auto make_b = [&](int box_rows, CUtensorMap *tb) {
    return make_tmap_2d(tb, Wq, CU_TENSOR_MAP_DATA_TYPE_UINT8, K, N, static_cast<uint64_t>(K),
                        kBKBytes, box_rows);
  };
  switch (out_type) {
    case ROUGE_B200_OUT_F32:
      return launch_tiles<MmaKind::I8, 256, false, ROUGE_B200_OUT_F32, false, true, true>(ta, make_b, g, st);
    case ROUGE_B200_OUT_BF16:
      return launch_tiles<MmaKind::I8, 256, false, ROUGE_B200_OUT_BF16, false, true, true>(ta, make_b, g, st);
    default:
      return launch_tiles<MmaKind::I8, 256, false, ROUGE_B200_OUT_I32, false, true, true>(ta, make_b, g, st);
  }
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
  g.vec16 = (reinterpret_cast<uintptr_t>(sb) & 15u) == 0;
  g.err = err;
  return launch_kind<MmaKind::I8>(A, lda, B, ldb, b_layout, g, out_type, st);
}

// The int8 GEMM with its output broadcast to every rank's C (see
// GemmArgs::bcast): the sharded W8A8 GEMM's all-gather fused into the
// epilogue.
int launch_gemm_i8_bcast(int M, int N, int K, const int8_t *A, long long lda, const int8_t *B,
                         long long ldb, int b_layout, const float *sa, int a_rows,
                         const float *sb, int b_cols, void *mc, void *const *peers, int npeers,
                         long long ldc, int col_off, int out_type, cudaStream_t st) {
  GemmArgs g{};
  g.M = M; g.N = N; g.K = K;
  g.scales_a = sa; g.scales_b = sb; g.a_rows = a_rows; g.b_cols = b_cols;
  g.use_tma_store = 0;
  g.vec16 = (reinterpret_cast<uintptr_t>(sb) & 15u) == 0;
  g.err = device_error_word();
  g.bcast = mc;
  g.npeers = mc ? 0 : npeers;
  for (int r = 0; r < g.npeers; ++r) g.peers[r] = peers[r];
  g.col_off = col_off;
  g.bld = ldc;
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

// BLAS-form GEMM on the f16 / bf16 / tf32 / e4m3 kinds:
// C[M][N] (f32, row pitch ldc) = alpha * A[M][K] . B^T + beta * C, A K-major
// (row pitch lda), B per b_layout (tf32 needs ROUGE_B200_B_NK).
// kind: 0 e4m3, 1 f16, 2 bf16, 3 tf32. tile_hint (kTileHint*) fixes the
// tile shape of this call; kTileHintAuto keeps the process-wide choice.
int launch_gemm_blas_tiles(int kind, int M, int N, int K, const void *A, long long lda,
                           const void *B, long long ldb, int b_layout, float alpha, float beta,
                           float *Cp, long long ldc, int tile_hint, cudaStream_t st) {
  if (tile_hint < kTileHintAuto || tile_hint > kTileHintPair) return set_status(ROUGE_B200_EINVAL);
  GemmArgs g{};
  g.tile_hint = tile_hint;
  g.M = M; g.N = N; g.K = K;
  g.C = Cp; g.ldc = ldc;
  g.blas = 1;
  g.alpha = alpha;
  g.beta = beta;
  g.bf16 = kind == 2 ? 1 : 0;
  g.use_tma_store = vec_ok(Cp, ldc, ROUGE_B200_OUT_F32);
  g.err = device_error_word();
  switch (kind) {
    case 0:
      return launch_kind<MmaKind::F8F6F4>(A, lda, B, ldb, b_layout, g, ROUGE_B200_OUT_F32, st);
    case 1:
    case 2:
      return launch_kind<MmaKind::F16>(A, lda, B, ldb, b_layout, g, ROUGE_B200_OUT_F32, st);
    case 3:
      if (b_layout != ROUGE_B200_B_NK) return set_status(ROUGE_B200_EUNSUPPORTED);
      return launch_kind<MmaKind::TF32>(A, lda, B, ldb, b_layout, g, ROUGE_B200_OUT_F32, st);
    default:
      return set_status(ROUGE_B200_EINVAL);
  }
}

int launch_gemm_blas(int kind, int M, int N, int K, const void *A, long long lda, const void *B,
                     long long ldb, int b_layout, float alpha, float beta, float *Cp,
                     long long ldc, cudaStream_t st) {
  return launch_gemm_blas_tiles(kind, M, N, K, A, lda, B, ldb, b_layout, alpha, beta, Cp, ldc,
                                kTileHintAuto, st);
}

// launch_gemm_blas over `batch` items stacked by rows (K-major B only):
// item i computes C[i*M + m][n] = alpha * sum_k A[i*M + m][k] B[i*N + n][k]
// (+ beta * C). M must be a multiple of 256 when batch > 1.
int launch_gemm_blas_batched(int kind, int M, int N, int K, const void *A, long long lda,
                             const void *B, long long ldb, float alpha, float beta, float *Cp,
                             long long ldc, int batch, cudaStream_t st) {
  if (batch <= 1)
    return launch_gemm_blas(kind, M, N, K, A, lda, B, ldb, ROUGE_B200_B_NK, alpha, beta, Cp, ldc,
                            st);
  if (M % 256 != 0 || kind != 3) return set_status(ROUGE_B200_EUNSUPPORTED);
  GemmArgs g{};
  g.M = M * batch; g.N = N; g.K = K;
  g.item_m = M;
  g.C = Cp; g.ldc = ldc;
  g.blas = 1;
  g.alpha = alpha;
  g.beta = beta;
  g.use_tma_store = vec_ok(Cp, ldc, ROUGE_B200_OUT_F32);
  g.err = device_error_word();
  return launch_kind<MmaKind::TF32>(A, lda, B, ldb, ROUGE_B200_B_NK, g, ROUGE_B200_OUT_F32, st);
}

// Block-scaled (MXFP8) GEMM on CTA pairs with 256 x 256 tiles:
// C[M][N] = sum_k (a[m][k] * 2^(sfa - 127)) (b[n][k] * 2^(sfb - 127)),
// f32 accumulation; A [M][K], B [N][K] e4m3 / e5m2 codes (row pitches lda,
// ldb bytes), scales in the tcgen05 atom layout (rouge_b200_mx_scale_atoms).
int launch_gemm_mx(int M, int N, int K, const uint8_t *A, long long lda, int fmt_a,
                   const uint8_t *sfa, const uint8_t *B, long long ldb, int fmt_b,
                   const uint8_t *sfb, void *Cp, long long ldc, int out_type, cudaStream_t st) {
  GemmArgs g{};
  g.M = M; g.N = N; g.K = K;
  g.C = Cp; g.ldc = ldc;
  g.scales_a = reinterpret_cast<const float *>(sfa);
  g.scales_b = reinterpret_cast<const float *>(sfb);
  g.mx_fmt_a = fmt_a;
  g.mx_fmt_b = fmt_b;
  g.sf_kblocks = (K + 127) / 128;
  g.use_tma_store = vec_ok(Cp, ldc, out_type);
  g.err = device_error_word();
  g.num_m = (M + 2 * kBM - 1) / (2 * kBM);
  g.num_n = (N + 255) / 256;
  g.num_k = (K + 127) / 128;
  g.num_tiles = g.num_m * g.num_n;
  if (out_type == ROUGE_B200_OUT_BF16)
    return launch_gemm_impl<MmaKind::MXF8, 256, false, ROUGE_B200_OUT_BF16, true>(A, lda, B, ldb, g,
                                                                                  st);
  return launch_gemm_impl<MmaKind::MXF8, 256, false, ROUGE_B200_OUT_F32, true>(A, lda, B, ldb, g,
                                                                               st);
}

// Block-scaled NVFP4 GEMM on CTA pairs, 256 x 256 tiles:
// C[M][N] = gs_a gs_b sum_k (a[m][k] * sa) (b[n][k] * sb), a / b packed
// e2m1 (two per byte, the lower-index element in the low nibble; row
// pitches K / 2 bytes), UE4M3 block scales per 16 K in the tcgen05 atom
// layout (rouge_b200_nvfp4_scale_atoms), gs_a / gs_b device floats or null.
template <MmaKind KIND>
int launch_gemm_fp4(int M, int N, int K, const uint8_t *A, const uint8_t *sfa, const float *gs_a,
                    const uint8_t *B, const uint8_t *sfb, const float *gs_b, void *Cp,
                    long long ldc, int out_type, cudaStream_t st) {
  GemmArgs g{};
  g.M = M; g.N = N; g.K = K;
  g.C = Cp; g.ldc = ldc;
  g.scales_a = reinterpret_cast<const float *>(sfa);
  g.scales_b = reinterpret_cast<const float *>(sfb);
  g.scale_a = gs_a && gs_b ? gs_a : nullptr;
  g.scale_b = gs_a && gs_b ? gs_b : nullptr;
  g.mx_fmt_a = 1;  // E2M1 of kind::mxf4nvf4 / kind::mxf4
  g.mx_fmt_b = 1;
  g.sf_kblocks = (K + 255) / 256;
  g.use_tma_store = vec_ok(Cp, ldc, out_type);
  g.err = device_error_word();
  g.num_m = (M + 2 * kBM - 1) / (2 * kBM);
  g.num_n = (N + 255) / 256;
  g.num_k = (K + 255) / 256;
  g.num_tiles = g.num_m * g.num_n;
  const uint64_t kbytes = static_cast<uint64_t>(K) / 2;
  CUtensorMap ta;
  int s = make_tmap_2d(&ta, A, CU_TENSOR_MAP_DATA_TYPE_UINT8, kbytes, M, kbytes, kBKBytes, kBM);
  if (s != ROUGE_B200_OK) return s;
  auto make_b = [&](int box_rows, CUtensorMap *tb) {
    return make_tmap_2d(tb, B, CU_TENSOR_MAP_DATA_TYPE_UINT8, kbytes, N, kbytes, kBKBytes, box_rows);
  };
  if (out_type == ROUGE_B200_OUT_BF16)
    return launch_tiles<KIND, 256, false, ROUGE_B200_OUT_BF16, false, true>(ta, make_b, g, st);
  return launch_tiles<KIND, 256, false, ROUGE_B200_OUT_F32, false, true>(ta, make_b, g, st);
}

}  // namespace rb200

using namespace rb200;

extern "C" {

int rouge_b200_gemm_nvfp4(int M, int N, int K, const uint8_t *A, const uint8_t *sfa,
                          const float *gs_a, const uint8_t *B, const uint8_t *sfb,
                          const float *gs_b, void *C, int ldc, int out_type, void *stream) {
  if (M <= 0 || N <= 0 || K <= 0 || !A || !B || !sfa || !sfb || !C || ldc < N ||
      (out_type != ROUGE_B200_OUT_F32 && out_type != ROUGE_B200_OUT_BF16))
    return set_status(ROUGE_B200_EINVAL);
  if (K % 32 || (reinterpret_cast<uintptr_t>(A) & 15u) || (reinterpret_cast<uintptr_t>(B) & 15u) ||
      (reinterpret_cast<uintptr_t>(sfa) & 15u) || (reinterpret_cast<uintptr_t>(sfb) & 15u))
    return set_status(ROUGE_B200_EUNSUPPORTED);
  const int s = device_ready();
  if (s != ROUGE_B200_OK) return s;
  return launch_gemm_fp4<MmaKind::NVF4>(M, N, K, A, sfa, gs_a, B, sfb, gs_b, C, ldc, out_type,
                                       as_stream(stream));
}

int rouge_b200_gemm_mxfp4(int M, int N, int K, const uint8_t *A, const uint8_t *sfa,
                          const uint8_t *B, const uint8_t *sfb, void *C, int ldc, int out_type,
                          void *stream) {
  if (M <= 0 || N <= 0 || K <= 0 || !A || !B || !sfa || !sfb || !C || ldc < N ||
      (out_type != ROUGE_B200_OUT_F32 && out_type != ROUGE_B200_OUT_BF16))
    return set_status(ROUGE_B200_EINVAL);
  if (K % 32 || (reinterpret_cast<uintptr_t>(A) & 15u) || (reinterpret_cast<uintptr_t>(B) & 15u) ||
      (reinterpret_cast<uintptr_t>(sfa) & 15u) || (reinterpret_cast<uintptr_t>(sfb) & 15u))
    return set_status(ROUGE_B200_EUNSUPPORTED);
  const int s = device_ready();
  if (s != ROUGE_B200_OK) return s;
  return launch_gemm_fp4<MmaKind::MXF4>(M, N, K, A, sfa, nullptr, B, sfb, nullptr, C, ldc, out_type,
                                        as_stream(stream));
}

int rouge_b200_gemm_mx(int M, int N, int K, const uint8_t *A, int fmt_a, const uint8_t *sfa,
                       const uint8_t *B, int fmt_b, const uint8_t *sfb, void *C, int ldc,
                       int out_type, void *stream) {
  if (M <= 0 || N <= 0 || K <= 0 || !A || !B || !sfa || !sfb || !C || ldc < N)
    return set_status(ROUGE_B200_EINVAL);
  if ((fmt_a != 0 && fmt_a != 1) || (fmt_b != 0 && fmt_b != 1) ||
      (out_type != ROUGE_B200_OUT_F32 && out_type != ROUGE_B200_OUT_BF16))
    return set_status(ROUGE_B200_EINVAL);
  if (K % 32 || (reinterpret_cast<uintptr_t>(A) & 15u) || (reinterpret_cast<uintptr_t>(B) & 15u) ||
      (reinterpret_cast<uintptr_t>(sfa) & 15u) || (reinterpret_cast<uintptr_t>(sfb) & 15u))
    return set_status(ROUGE_B200_EUNSUPPORTED);
  const int s = device_ready();
  if (s != ROUGE_B200_OK) return s;
  return launch_gemm_mx(M, N, K, A, K, fmt_a, sfa, B, K, fmt_b, sfb, C, ldc, out_type,
                        as_stream(stream));
}

int rouge_b200_set_clock_probe(unsigned long long *stamps, int ctas) {
  if (ctas < 0) return set_status(ROUGE_B200_EINVAL);
  if (!stamps || ctas == 0) {
    g_clock_stamps.store(nullptr);
    return ROUGE_B200_OK;
  }
  g_clock_dev.store(current_device());
  g_clock_ctas.store(ctas);
  g_clock_stamps.store(stamps);
  return ROUGE_B200_OK;
}

int rouge_b200_set_tile_mode(int mode) {
  if (mode != ROUGE_B200_TILES_AUTO && mode != ROUGE_B200_TILES_SINGLE &&
      mode != ROUGE_B200_TILES_PAIR)
    return set_status(ROUGE_B200_EINVAL);
  return g_tile_mode.exchange(mode);
}

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

size_t rouge_b200_w8a8_workspace_bytes(int M) {
  return M > 0 ? (static_cast<size_t>(M + 127) / 128 + 2) * sizeof(unsigned) : 0;
}

int rouge_b200_w8a8_linear(int M, int N, int K, const float *X, const int8_t *Wq, const float *sw,
                           int8_t *Aq, float *sa, void *C, int ldc, int out_type, void *workspace,
                           void *stream) {
  if (!X || !sw || !sa || !workspace) return set_status(ROUGE_B200_EINVAL);
  int s = check_common(M, N, K, Aq, Wq, C, ldc, ROUGE_B200_B_NK, out_type, 1);
  if (s != ROUGE_B200_OK) return set_status(s);
  if ((K & 3) || (reinterpret_cast<uintptr_t>(X) & 15u) || (reinterpret_cast<uintptr_t>(workspace) & 3u))
    return set_status(ROUGE_B200_EUNSUPPORTED);
  s = device_ready();
  if (s != ROUGE_B200_OK) return s;
  return launch_w8a8_linear(M, N, K, X, Wq, sw, Aq, sa, C, ldc, out_type,
                            static_cast<unsigned *>(workspace), as_stream(stream));
}

int rouge_b200_gemm_i8_bcast(int M, int N, int K, const int8_t *A, const int8_t *B, int b_layout,
                             const float *scales_a, int a_rows, const float *scales_b, int b_cols,
                             void *C_mc, void *const *C_peers, int npeers, long long ldc,
                             int col_off, int out_type, void *stream) {
  if (M <= 0 || N <= 0 || K <= 0 || !A || !B || col_off < 0 || ldc < static_cast<long long>(col_off) + N)
    return set_status(ROUGE_B200_EINVAL);
  if (b_layout != ROUGE_B200_B_KN && b_layout != ROUGE_B200_B_NK) return set_status(ROUGE_B200_EINVAL);
  if (out_type != ROUGE_B200_OUT_F32 && out_type != ROUGE_B200_OUT_BF16 &&
      out_type != ROUGE_B200_OUT_I32)
    return set_status(ROUGE_B200_EINVAL);
  if (out_type != ROUGE_B200_OUT_I32 && (!scales_a || !scales_b)) return set_status(ROUGE_B200_EINVAL);
  if (!C_mc && (!C_peers || npeers < 1 || npeers > 8)) return set_status(ROUGE_B200_EINVAL);
  const long long esz = out_type == ROUGE_B200_OUT_BF16 ? 2 : 4;
  // 16-byte vectors: row pitch, column offset and width in whole vectors.
  if ((ldc * esz) % 16 || (col_off * esz) % 16 || N % 8 || K % 16 ||
      (b_layout == ROUGE_B200_B_KN && N % 16) ||
      (reinterpret_cast<uintptr_t>(A) & 15u) || (reinterpret_cast<uintptr_t>(B) & 15u) ||
      (reinterpret_cast<uintptr_t>(C_mc) & 15u))
    return set_status(ROUGE_B200_EUNSUPPORTED);
  if (!C_mc)
    for (int r = 0; r < npeers; ++r)
      if (!C_peers[r] || (reinterpret_cast<uintptr_t>(C_peers[r]) & 15u))
        return set_status(ROUGE_B200_EINVAL);
  int s = device_ready();
  if (s != ROUGE_B200_OK) return s;
  const long long ldb = b_layout == ROUGE_B200_B_KN ? N : K;
  return launch_gemm_i8_bcast(M, N, K, A, K, B, ldb, b_layout, scales_a, a_rows, scales_b, b_cols,
                              C_mc, C_peers, npeers, ldc, col_off, out_type, as_stream(stream));
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
