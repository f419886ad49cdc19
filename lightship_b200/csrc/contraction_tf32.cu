// contraction_tf32.cu -- FP32 contractions on the 5th-generation tensor cores as
// split-TF32 (three tcgen05.mma.kind::tf32 products per K slice: hi*hi + hi*lo + lo*hi, f32
// accumulation in TMEM), or plain TF32 (one product) when the caller asks for it.
//   * GEMM  C[M,N] = A[M,K] B[N,K]^T (+ bias[n], activation)  -- MatMul (B transposed by the
//     prep kernel) and FullyConnected (lightship-core/src/backend/cpu.rs:949-1063, :1209-1290)
//   * Conv2d as an implicit GEMM over NHWC operands with TMA im2col loads, output written
//     back as NCHW, folded BatchNorm / bias / ReLU / ReLU6 / SiLU in the epilogue
//     (core/operator/convolution.rs:90-267, cpu.rs:277-439, core/ir/optimizer.rs:727-731).
// Pipeline and warp roles follow contraction_i8.cu: warp 0 TMA producer, warp 1 MMA issuer,
// warps 2-9 epilogue, double-buffered TMEM accumulators, bounded mbarrier waits.
#include <mutex>

#include "epilogue.cuh"
#include "lsc_internal.h"
#include "sm100.cuh"

namespace lsc {
namespace {

struct Tf32Params {
  int32_t m, n, k;  // GEMM view: rows, output channels, K in f32 elements (multiple of 32 stages)
  const float* bias;
  int32_t act;
  float* out;
  int64_t ldo;       // row-major output stride (GEMM)
  int32_t out_nchw;  // convolution: write out[(img * n + col) * ohw + pix]
  int32_t vec_ok;
  uint32_t* err;
  int32_t ow, ohw, sw, sh, pw, ph, dw, dh, kw;
  int32_t chunks_per_tap, total_chunks, chunk_elems;
  // batched GEMM (GEMM mode only): `batches` independent products; batch b's A rows start at
  // b * a_batch_rows of A's tensor map, its B rows at b * b_batch_rows, its output at
  // out + b * out_batch_stride.  Rows or columns a tile reads past its batch's m / n belong
  // to the next batch (or lie past the map, zero-filled) and are never stored.
  int32_t batches, a_batch_rows, b_batch_rows;
  int64_t out_batch_stride;
  // split K (one batch only): ksplit CTAs share a tile, each over kb_per_split K blocks, and
  // write their raw f32 sums to partial[split][m][n]; tf32_splitk_reduce adds them in order
  int32_t ksplit, kb_per_split;
  float* partial;
};

template <int BN_, bool SPLIT_>
struct Tf32Cfg {
  static constexpr int BM = 128;
  static constexpr int BN = BN_;
  static constexpr int BK = 32;  // f32 elements of K per stage (128 bytes)
  static constexpr int PARTS = SPLIT_ ? 2 : 1;
  static constexpr int A_PART = BM * 128;
  static constexpr int B_PART = BN * 128;
  static constexpr int STAGE_BYTES = PARTS * (A_PART + B_PART);
  static constexpr int STAGES = (196608 / STAGE_BYTES) < 8 ? (196608 / STAGE_BYTES) : 8;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int EPI_WARPS = 8;
  static constexpr int THREADS = 64 + 32 * EPI_WARPS;
  static constexpr int COLS_PER_EPI_WARP = BN / 2;
  static constexpr int BAR_BYTES = 256;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + BAR_BYTES;
  static constexpr uint32_t IDESC = idesc_tf32(BM, BN, 0);
  static_assert(STAGES >= 2, "pipeline depth");
  static_assert(SMEM_BYTES <= 232448, "shared memory budget");
  static_assert((2 * STAGES + 5) * 8 + 8 <= BAR_BYTES, "barrier area");
};

// A-operand descriptor of K slice kk (32 bytes) -- same sub-tile geometry as the INT8 kernel.
template <int ACB>
__device__ __forceinline__ uint64_t a_desc(uint32_t a0, int kk) {
  if constexpr (ACB == 0 || ACB == 128) {
    return smem_desc_sw128_kmajor(a0 + kk * 32);
  } else if constexpr (ACB == 64) {
    return smem_desc_sw64_kmajor(a0 + (kk >> 1) * (128 * 64) + (kk & 1) * 32);
  } else if constexpr (ACB == 32) {
    return smem_desc_sw32_kmajor(a0 + kk * (128 * 32));
  } else {
    static_assert(ACB == 16, "channel block must be 16, 32, 64 or 128 bytes");
    return smem_desc_noswz_kmajor(a0 + kk * 2 * (128 * 16), 128 * 16, 128);
  }
}

__device__ __forceinline__ float act_rt(float x, int act) {
  switch (act) {
    case LSC_ACT_RELU: return act_relu(x);
    case LSC_ACT_RELU6: return act_relu6(x);
    case LSC_ACT_SILU: return act_silu(x);
    case LSC_ACT_GELU: return act_gelu(x);
    default: return x;
  }
}

template <int BN, int ACB, bool SPLIT>
__global__ void __launch_bounds__(Tf32Cfg<BN, SPLIT>::THREADS, 1)
    contraction_tf32_kernel(const __grid_constant__ CUtensorMap tmAh,
                            const __grid_constant__ CUtensorMap tmAl,
                            const __grid_constant__ CUtensorMap tmBh,
                            const __grid_constant__ CUtensorMap tmBl, const Tf32Params p) {
  using C = Tf32Cfg<BN, SPLIT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::STAGES * C::STAGE_BYTES);
  uint64_t* full = bars;
  uint64_t* empty = bars + C::STAGES;
  uint64_t* tfull = bars + 2 * C::STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile uint32_t* abort_flag = tmem_slot + 1;
  // stage layout: [A hi][A lo][B hi][B lo]
  auto a_part = [&](int stage, int part) { return smem + stage * C::STAGE_BYTES + part * C::A_PART; };
  auto b_part = [&](int stage, int part) {
    return smem + stage * C::STAGE_BYTES + C::PARTS * C::A_PART + part * C::B_PART;
  };

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], C::EPI_WARPS);
    }
    mbar_init(drain, 1);
    *abort_flag = 0u;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmAh);
    tma_prefetch_desc(&tmBh);
    if constexpr (SPLIT) {
      tma_prefetch_desc(&tmAl);
      tma_prefetch_desc(&tmBl);
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  griddep_wait();  // launched as a dependent kernel: operands and outputs are settled from here on
  griddep_launch_dependents();

  const int m_tiles = (p.m + C::BM - 1) / C::BM;
  const int n_tiles = (p.n + C::BN - 1) / C::BN;
  const int batch_tiles = m_tiles * n_tiles;
  const int out_tiles = batch_tiles * p.batches;
  const int num_tiles = out_tiles * p.ksplit;
  const int kblocks = (p.k + C::BK - 1) / C::BK;

  if (warp == 0) {
    if (lane == 0) {
      uint32_t stage = 0, phase = 0;
      int issued = 0;
      bool ok = true;
      for (int tile_k = blockIdx.x; tile_k < num_tiles && ok; tile_k += gridDim.x) {
        const int ks = tile_k / out_tiles, tile = tile_k - ks * out_tiles;
        const int kb0 = ks * p.kb_per_split;
        const int kb1 = kb0 + p.kb_per_split < kblocks ? kb0 + p.kb_per_split : kblocks;
        const int bz = tile / batch_tiles;
        const int mb = (tile - bz * batch_tiles) % m_tiles, nb = (tile - bz * batch_tiles) / m_tiles;
        const int a_row0 = bz * p.a_batch_rows + mb * C::BM, b_row0 = bz * p.b_batch_rows + nb * C::BN;
        int32_t cw = 0, chh = 0, cn = 0;
        if constexpr (ACB > 0) {
          const int m0 = mb * C::BM;
          cn = m0 / p.ohw;
          const int rem = m0 - cn * p.ohw;
          const int oy = rem / p.ow;
          const int ox = rem - oy * p.ow;
          cw = ox * p.sw - p.pw;
          chh = oy * p.sh - p.ph;
        }
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, p.err)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
#pragma unroll
          for (int part = 0; part < C::PARTS; ++part) {
            const CUtensorMap* ta = part == 0 ? &tmAh : &tmAl;
            const CUtensorMap* tb = part == 0 ? &tmBh : &tmBl;
            if constexpr (ACB == 0) {
              tma_load_2d(ta, &full[stage], a_part(stage, part), kb * C::BK, a_row0);
            } else {
              constexpr int SUB = 128 / ACB;
#pragma unroll
              for (int i = 0; i < SUB; ++i) {
                int j = kb * SUB + i;
                if (j >= p.total_chunks) j = 0;  // past the filter: weights are zero there
                const int tap = j / p.chunks_per_tap;
                const int c0 = (j - tap * p.chunks_per_tap) * p.chunk_elems;
                const int ky = tap / p.kw;
                const int kx = tap - ky * p.kw;
                tma_load_im2col_4d(ta, &full[stage], a_part(stage, part) + i * (C::BM * ACB), c0, cw,
                                   chh, cn, static_cast<uint16_t>(kx * p.dw),
                                   static_cast<uint16_t>(ky * p.dh));
              }
            }
            tma_load_2d(tb, &full[stage], b_part(stage, part), kb * C::BK, b_row0);
          }
          ++issued;
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        volatile uint32_t no_abort = 0;
        const int outstanding = issued < C::STAGES ? issued : C::STAGES;
        for (int i = 1; i <= outstanding; ++i) {
          const int idx = issued - i;
          mbar_wait(&full[idx % C::STAGES], static_cast<uint32_t>((idx / C::STAGES) & 1), &no_abort,
                    p.err);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      uint32_t stage = 0, phase = 0;
      int local = 0;
      bool ok = true, any_mma = false;
      for (int tile_k = blockIdx.x; tile_k < num_tiles && ok; tile_k += gridDim.x, ++local) {
        const int kb0 = (tile_k / out_tiles) * p.kb_per_split;
        const int kb1 = kb0 + p.kb_per_split < kblocks ? kb0 + p.kb_per_split : kblocks;
        const int buf = local & 1;
        const uint32_t buf_phase = static_cast<uint32_t>((local >> 1) & 1);
        if (!mbar_wait(&tempty[buf], buf_phase ^ 1u, abort_flag, p.err)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * C::BN);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, p.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t ah = smem_u32(a_part(stage, 0));
          const uint32_t bh = smem_u32(b_part(stage, 0));
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t adh = a_desc<ACB>(ah, kk);
            const uint64_t bdh = smem_desc_sw128_kmajor(bh + kk * 32);
            mma_tf32(d_tmem, adh, bdh, C::IDESC, (kb != kb0 || kk != 0) ? 1u : 0u);
            if constexpr (SPLIT) {
              const uint64_t adl = a_desc<ACB>(smem_u32(a_part(stage, 1)), kk);
              const uint64_t bdl = smem_desc_sw128_kmajor(smem_u32(b_part(stage, 1)) + kk * 32);
              mma_tf32(d_tmem, adh, bdl, C::IDESC, 1u);
              mma_tf32(d_tmem, adl, bdh, C::IDESC, 1u);
            }
          }
          any_mma = true;
          mma_commit(&empty[stage]);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (ok) mma_commit(&tfull[buf]);
      }
      if (!ok && any_mma) {
        volatile uint32_t no_abort = 0;
        mma_commit(drain);
        mbar_wait(drain, 0u, &no_abort, p.err);
      }
    }
  } else {
    const int epi = warp - 2;
    const int quarter = warp & 3;
    const int half = epi >> 2;
    const int row_in_tile = quarter * 32 + lane;
    int local = 0;
    for (int tile_k = blockIdx.x; tile_k < num_tiles; tile_k += gridDim.x, ++local) {
      const int ks = tile_k / out_tiles, tile = tile_k - ks * out_tiles;
      const int bz = tile / batch_tiles;
      const int mb = (tile - bz * batch_tiles) % m_tiles, nb = (tile - bz * batch_tiles) / m_tiles;
      float* const out_b = p.out + bz * p.out_batch_stride;
      const int buf = local & 1;
      const uint32_t buf_phase = static_cast<uint32_t>((local >> 1) & 1);
      if (!mbar_wait(&tfull[buf], buf_phase, abort_flag, p.err)) break;
      tc_fence_after();
      const int row = mb * C::BM + row_in_tile;
      constexpr int CHUNKS = C::COLS_PER_EPI_WARP / 32;
#pragma unroll 1
      for (int c = 0; c < CHUNKS; ++c) {
        const int tcol = half * C::COLS_PER_EPI_WARP + c * 32;
        const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                               static_cast<uint32_t>(buf * C::BN + tcol);
        uint32_t r[32];
        tmem_ld_32x32b_x32(taddr, r);
        tmem_ld_wait();
        if (c == CHUNKS - 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tempty[buf]);
        }
        if (row >= p.m) continue;
        const int col0 = nb * C::BN + tcol;
        if (p.ksplit > 1) {  // raw sums of this K range; bias and activation after the reduction
          float* o = p.partial + (static_cast<int64_t>(ks) * p.m + row) * p.n + col0;
          if (p.n % 4 == 0 && col0 + 32 <= p.n) {
#pragma unroll
            for (int j = 0; j < 8; ++j)
              reinterpret_cast<float4*>(o)[j] = make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                                                            __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (col0 + j < p.n) o[j] = __uint_as_float(r[j]);
          }
          continue;
        }
        float y[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int col = col0 + j;
          float v = __uint_as_float(r[j]);
          if (p.bias && col < p.n) v = __fadd_rn(v, __ldg(p.bias + col));
          y[j] = act_rt(v, p.act);
        }
        if (p.out_nchw) {
          const int img = row / p.ohw;
          const int pix = row - img * p.ohw;
          float* o = out_b + (static_cast<int64_t>(img) * p.n + col0) * p.ohw + pix;
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (col0 + j < p.n) o[static_cast<int64_t>(j) * p.ohw] = y[j];
        } else {
          float* o = out_b + static_cast<int64_t>(row) * p.ldo + col0;
          if (p.vec_ok && col0 + 32 <= p.n) {
#pragma unroll
            for (int j = 0; j < 8; ++j)
              reinterpret_cast<float4*>(o)[j] = make_float4(y[4 * j], y[4 * j + 1], y[4 * j + 2], y[4 * j + 3]);
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (col0 + j < p.n) o[j] = y[j];
          }
        }
      }
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// out = act(sum over the K splits, in split order, + bias): row-major [m, ldo] or, for a
// convolution, NCHW (element i walks the NCHW output so that the stores coalesce).
__global__ void tf32_splitk_reduce_kernel(const float* __restrict__ partial, int32_t ksplit, int32_t m, int32_t n,
                                          const float* __restrict__ bias, int32_t act, float* __restrict__ out,
                                          int64_t ldo, int32_t out_nchw, int32_t ohw) {
  griddep_wait();  // launched as a dependent kernel: the partial sums are complete from here on
  griddep_launch_dependents();
  const int64_t total = static_cast<int64_t>(m) * n;
  const int64_t mn = total;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    int64_t row, col;
    if (out_nchw) {
      const int64_t img = i / (static_cast<int64_t>(n) * ohw);
      const int64_t rem = i - img * n * ohw;
      col = rem / ohw;
      row = img * ohw + (rem - col * ohw);
    } else {
      row = i / n;
      col = i - row * n;
    }
    float v = partial[row * n + col];
    for (int s = 1; s < ksplit; ++s) v = __fadd_rn(v, partial[s * mn + row * n + col]);
    if (bias) v = __fadd_rn(v, __ldg(bias + col));
    v = act_rt(v, act);
    if (out_nchw) out[i] = v;
    else out[row * ldo + col] = v;
  }
}

template <int BN, int ACB, bool SPLIT>
lsc_status launch_cfg(const CUtensorMap (&tm)[4], const Tf32Params& p, int sm_count, bool overlap,
                      cudaStream_t stream) {
  using C = Tf32Cfg<BN, SPLIT>;
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [] {
    attr_err = cudaFuncSetAttribute(contraction_tf32_kernel<BN, ACB, SPLIT>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
  });
  if (attr_err != cudaSuccess) return cuda_error(attr_err, "cudaFuncSetAttribute(contraction_tf32)");
  const int64_t tiles =
      static_cast<int64_t>((p.m + C::BM - 1) / C::BM) * ((p.n + C::BN - 1) / C::BN) * p.batches * p.ksplit;
  const int grid = tiles < sm_count ? static_cast<int>(tiles) : sm_count;
  LSC_CUDA_TRY(launch_dependent(overlap, contraction_tf32_kernel<BN, ACB, SPLIT>, dim3(grid), dim3(C::THREADS),
                                static_cast<size_t>(C::SMEM_BYTES), stream, tm[0], tm[1], tm[2], tm[3], p));
  if (p.ksplit > 1) {
    const int64_t total = static_cast<int64_t>(p.m) * p.n;
    const int64_t blocks = (total + 255) / 256;
    const int rgrid = static_cast<int>(blocks < 8 * sm_count ? blocks : 8 * sm_count);
    LSC_CUDA_TRY(launch_dependent(overlap, tf32_splitk_reduce_kernel, dim3(rgrid), dim3(256), 0, stream, p.partial,
                                  p.ksplit, p.m, p.n, p.bias, p.act, p.out, p.ldo, p.out_nchw, p.ohw));
  }
  return LSC_SUCCESS;
}

template <int ACB>
lsc_status launch_acb(int bn, bool split, const CUtensorMap (&tm)[4], const Tf32Params& p,
                      int sm_count, cudaStream_t stream) {
  const DeviceState* ds = current_device_state();
  const bool overlap = ds ? ds->overlap_launches : false;
  if (bn == 64)
    return split ? launch_cfg<64, ACB, true>(tm, p, sm_count, overlap, stream)
                 : launch_cfg<64, ACB, false>(tm, p, sm_count, overlap, stream);
  return split ? launch_cfg<128, ACB, true>(tm, p, sm_count, overlap, stream)
               : launch_cfg<128, ACB, false>(tm, p, sm_count, overlap, stream);
}

lsc_status check_ptr16(const void* p, const char* what) {
  if (reinterpret_cast<uintptr_t>(p) & 15)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "%s must be 16-byte aligned", what);
  return LSC_SUCCESS;
}

// K splits for a product of `tiles` output tiles and `kblocks` K blocks: none while the tiles
// fill half the SMs; else up to one CTA per SM, at least two K blocks each, at most 16 splits.
// A single producer thread issues each CTA's tensor loads one after another, so a small
// product with a long K runs at the pace of its few CTAs' load streams (the 512^3 GEMM on 16
// CTAs, a batch-1 56x56 convolution on 25) unless K is spread over more CTAs.
void choose_ksplit(int64_t tiles, int64_t kblocks, int sm_count, int32_t& ksplit, int32_t& kb_per_split) {
  ksplit = 1;
  kb_per_split = static_cast<int32_t>(kblocks);
  if (tiles <= 0 || 2 * tiles > sm_count || kblocks < 4) return;
  int64_t s = sm_count / tiles;
  if (s > kblocks / 2) s = kblocks / 2;
  if (s > 16) s = 16;
  if (s < 2) return;
  const int64_t per = (kblocks + s - 1) / s;
  ksplit = static_cast<int32_t>((kblocks + per - 1) / per);
  kb_per_split = static_cast<int32_t>(per);
}

int64_t gemm_tiles(int64_t m, int64_t n, int64_t batches) {
  const int64_t bn = n <= 64 ? 64 : 128;
  return ((m + 127) / 128) * ((n + bn - 1) / bn) * batches;
}

int64_t conv_kblocks(const ConvGeometry& g) {
  const int64_t cbytes = g.c * 4;
  const int64_t acb = cbytes % 128 == 0 ? 128 : (cbytes % 64 == 0 ? 64 : (cbytes % 32 == 0 ? 32 : 16));
  const int64_t total_chunks = g.kh * g.kw * (cbytes / acb);
  const int64_t sub = 128 / acb;
  return (total_chunks + sub - 1) / sub;
}

}  // namespace

int64_t tf32_gemm_ksplit_floats(int64_t m, int64_t n, int64_t k) {
  DeviceState* ds = current_device_state();
  if (!ds || m <= 0 || n <= 0 || k <= 0) return 0;
  int32_t ks = 1, per = 0;
  choose_ksplit(gemm_tiles(m, n, 1), (k + 31) / 32, ds->sm_count, ks, per);
  return ks > 1 ? ks * m * n : 0;
}

int64_t tf32_conv_ksplit_floats(const ConvGeometry& g) {
  DeviceState* ds = current_device_state();
  const int64_t m = g.n * g.oh * g.ow;
  if (!ds || m <= 0 || g.c_out <= 0 || g.c <= 0) return 0;
  int32_t ks = 1, per = 0;
  choose_ksplit(gemm_tiles(m, g.c_out, 1), conv_kblocks(g), ds->sm_count, ks, per);
  return ks > 1 ? ks * m * g.c_out : 0;
}

lsc_status launch_gemm_tf32_batched(const float* a_hi, const float* a_lo, const float* b_hi,
                                    const float* b_lo, int64_t batches, int64_t m, int64_t n, int64_t k,
                                    const float* bias, int act, float* out, int64_t ldo,
                                    int64_t out_batch_stride, bool split, cudaStream_t stream,
                                    float* ksplit_ws, int64_t ksplit_ws_floats) {
  if (m < 0 || n < 0 || k < 0 || batches < 0) return set_error(LSC_ERROR_INVALID_ARGUMENT, "gemm_tf32: negative size");
  if (m == 0 || n == 0 || batches == 0) return LSC_SUCCESS;
  if (!a_hi || !b_hi || !out || (split && (!a_lo || !b_lo)))
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "gemm_tf32: null operand");
  if (k == 0 || k % 4 != 0)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "gemm_tf32: K must be a positive multiple of 4");
  if (batches * m > INT32_MAX / 2 || batches * n > INT32_MAX / 2 || k > INT32_MAX / 2)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "gemm_tf32: size too large");
  if (act < LSC_ACT_NONE || act > LSC_ACT_GELU) return set_error(LSC_ERROR_INVALID_ARGUMENT, "gemm_tf32: bad activation");
  lsc_status st;
  if ((st = check_ptr16(a_hi, "A")) || (st = check_ptr16(b_hi, "B")) ||
      (split && ((st = check_ptr16(a_lo, "A lo")) || (st = check_ptr16(b_lo, "B lo")))))
    return st;
  DeviceState* ds = current_device_state();
  if (!ds) return LSC_ERROR_DEVICE_ERROR;
  if (ds->cc_major != 10) return set_error(LSC_ERROR_BACKEND_NOT_AVAILABLE, "gemm_tf32: needs sm_100");
  const int bn = n <= 64 ? 64 : 128;
  CUtensorMap tm[4];
  const float* srcs[4] = {a_hi, split ? a_lo : a_hi, b_hi, split ? b_lo : b_hi};
  for (int i = 0; i < 4; ++i) {
    const bool is_a = i < 2;
    st = encode_tmap_2d(&tm[i], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, srcs[i], k, batches * (is_a ? m : n), k * 4, 32,
                        is_a ? 128 : bn, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
  }
  Tf32Params p{};
  p.m = static_cast<int32_t>(m);
  p.n = static_cast<int32_t>(n);
  p.k = static_cast<int32_t>(k);
  p.bias = bias;
  p.act = act;
  p.out = out;
  p.ldo = ldo;
  p.out_nchw = 0;
  p.vec_ok = ((reinterpret_cast<uintptr_t>(out) & 15) == 0 && ldo % 4 == 0 && out_batch_stride % 4 == 0) ? 1 : 0;
  p.err = ds->err_word;
  p.batches = static_cast<int32_t>(batches);
  p.a_batch_rows = static_cast<int32_t>(m);
  p.b_batch_rows = static_cast<int32_t>(n);
  p.out_batch_stride = out_batch_stride;
  p.ksplit = 1;
  p.kb_per_split = static_cast<int32_t>((k + 31) / 32);
  if (ksplit_ws && batches == 1) {
    int32_t ks = 1, per = 0;
    choose_ksplit(gemm_tiles(m, n, 1), (k + 31) / 32, ds->sm_count, ks, per);
    if (ks > 1 && ks * m * n <= ksplit_ws_floats) {
      p.ksplit = ks;
      p.kb_per_split = per;
      p.partial = ksplit_ws;
    }
  }
  return launch_acb<0>(bn, split, tm, p, ds->sm_count, stream);
}

lsc_status launch_gemm_tf32(const float* a_hi, const float* a_lo, const float* b_hi,
                            const float* b_lo, int64_t m, int64_t n, int64_t k,
                            const float* bias, int act, float* out, int64_t ldo, bool split,
                            cudaStream_t stream, float* ksplit_ws, int64_t ksplit_ws_floats) {
  return launch_gemm_tf32_batched(a_hi, a_lo, b_hi, b_lo, 1, m, n, k, bias, act, out, ldo, 0, split, stream,
                                  ksplit_ws, ksplit_ws_floats);
}

lsc_status launch_conv_tf32(const float* x_hi, const float* x_lo, const float* w_hi,
                            const float* w_lo, const ConvGeometry& g, const float* bias, int act,
                            float* out_nchw, bool split, cudaStream_t stream, float* ksplit_ws,
                            int64_t ksplit_ws_floats) {
  const int64_t m = g.n * g.oh * g.ow;
  if (g.n < 0 || g.h <= 0 || g.w <= 0 || g.c <= 0 || g.kh <= 0 || g.kw <= 0 || g.sh <= 0 ||
      g.sw <= 0 || g.dh <= 0 || g.dw <= 0 || g.ph < 0 || g.pw < 0 || g.c_out < 0)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "conv_tf32: bad geometry");
  if (g.oh != (g.h + 2 * g.ph - g.dh * (g.kh - 1) - 1) / g.sh + 1 ||
      g.ow != (g.w + 2 * g.pw - g.dw * (g.kw - 1) - 1) / g.sw + 1 || g.oh <= 0 || g.ow <= 0)
    return set_error(LSC_ERROR_SHAPE_MISMATCH, "conv_tf32: output size does not match the geometry");
  if (g.c % 4 != 0) return set_error(LSC_ERROR_INVALID_ARGUMENT, "conv_tf32: stored channels must be a multiple of 4");
  if (g.sh > 8 || g.sw > 8 || g.ph > 127 || g.pw > 127 || g.ph - (g.kh - 1) * g.dh < -128 ||
      g.pw - (g.kw - 1) * g.dw < -128)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "conv_tf32: stride/padding outside the im2col unit's range");
  if (m == 0 || g.c_out == 0) return LSC_SUCCESS;
  if (m > INT32_MAX / 2) return set_error(LSC_ERROR_INVALID_ARGUMENT, "conv_tf32: problem too large");
  if (!x_hi || !w_hi || !out_nchw || (split && (!x_lo || !w_lo)))
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "conv_tf32: null operand");
  lsc_status st;
  if ((st = check_ptr16(x_hi, "x")) || (st = check_ptr16(w_hi, "w")) ||
      (split && ((st = check_ptr16(x_lo, "x lo")) || (st = check_ptr16(w_lo, "w lo")))))
    return st;
  if (act < LSC_ACT_NONE || act > LSC_ACT_GELU) return set_error(LSC_ERROR_INVALID_ARGUMENT, "conv_tf32: bad activation");
  DeviceState* ds = current_device_state();
  if (!ds) return LSC_ERROR_DEVICE_ERROR;
  if (ds->cc_major != 10) return set_error(LSC_ERROR_BACKEND_NOT_AVAILABLE, "conv_tf32: needs sm_100");

  const int64_t cbytes = g.c * 4;
  const int acb = cbytes % 128 == 0 ? 128 : (cbytes % 64 == 0 ? 64 : (cbytes % 32 == 0 ? 32 : 16));
  const int64_t k = g.kh * g.kw * g.c;  // elements
  const uint64_t dims[4] = {static_cast<uint64_t>(g.c), static_cast<uint64_t>(g.w),
                            static_cast<uint64_t>(g.h), static_cast<uint64_t>(g.n)};
  const uint64_t strides[3] = {static_cast<uint64_t>(g.c * 4), static_cast<uint64_t>(g.w * g.c * 4),
                               static_cast<uint64_t>(g.h * g.w * g.c * 4)};
  const int lower[2] = {static_cast<int>(-g.pw), static_cast<int>(-g.ph)};
  const int upper[2] = {static_cast<int>(g.pw - (g.kw - 1) * g.dw),
                        static_cast<int>(g.ph - (g.kh - 1) * g.dh)};
  const uint32_t estr[4] = {1, static_cast<uint32_t>(g.sw), static_cast<uint32_t>(g.sh), 1};
  const CUtensorMapSwizzle swz = acb == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                 : acb == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                 : acb == 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                                             : CU_TENSOR_MAP_SWIZZLE_NONE;
  const int bn = g.c_out <= 64 ? 64 : 128;
  CUtensorMap tm[4];
  const float* xs[2] = {x_hi, split ? x_lo : x_hi};
  const float* ws[2] = {w_hi, split ? w_lo : w_hi};
  for (int i = 0; i < 2; ++i) {
    st = encode_tmap_im2col(&tm[i], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, xs[i], dims, strides, lower, upper,
                            static_cast<uint32_t>(acb / 4), 128, estr, swz);
    if (st) return st;
    st = encode_tmap_2d(&tm[2 + i], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, ws[i], static_cast<uint64_t>(k),
                        static_cast<uint64_t>(g.c_out), static_cast<uint64_t>(k * 4), 32, bn,
                        CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
  }
  Tf32Params p{};
  p.m = static_cast<int32_t>(m);
  p.n = static_cast<int32_t>(g.c_out);
  const int64_t chunks_per_tap = cbytes / acb;
  const int64_t total_chunks = g.kh * g.kw * chunks_per_tap;
  const int64_t sub = 128 / acb;
  p.k = static_cast<int32_t>(((total_chunks + sub - 1) / sub) * 32);
  p.bias = bias;
  p.act = act;
  p.out = out_nchw;
  p.ldo = 0;
  p.out_nchw = 1;
  p.vec_ok = 0;
  p.err = ds->err_word;
  p.ow = static_cast<int32_t>(g.ow);
  p.ohw = static_cast<int32_t>(g.oh * g.ow);
  p.sw = static_cast<int32_t>(g.sw);
  p.sh = static_cast<int32_t>(g.sh);
  p.pw = static_cast<int32_t>(g.pw);
  p.ph = static_cast<int32_t>(g.ph);
  p.dw = static_cast<int32_t>(g.dw);
  p.dh = static_cast<int32_t>(g.dh);
  p.kw = static_cast<int32_t>(g.kw);
  p.chunks_per_tap = static_cast<int32_t>(chunks_per_tap);
  p.total_chunks = static_cast<int32_t>(total_chunks);
  p.chunk_elems = acb / 4;
  p.batches = 1;
  p.ksplit = 1;
  p.kb_per_split = static_cast<int32_t>(conv_kblocks(g));
  if (ksplit_ws) {
    int32_t ks = 1, per = 0;
    choose_ksplit(gemm_tiles(m, g.c_out, 1), conv_kblocks(g), ds->sm_count, ks, per);
    if (ks > 1 && ks * m * g.c_out <= ksplit_ws_floats) {
      p.ksplit = ks;
      p.kb_per_split = per;
      p.partial = ksplit_ws;
    }
  }
  switch (acb) {
    case 128: return launch_acb<128>(bn, split, tm, p, ds->sm_count, stream);
    case 64: return launch_acb<64>(bn, split, tm, p, ds->sm_count, stream);
    case 32: return launch_acb<32>(bn, split, tm, p, ds->sm_count, stream);
    default: return launch_acb<16>(bn, split, tm, p, ds->sm_count, stream);
  }
}

}  // namespace lsc
