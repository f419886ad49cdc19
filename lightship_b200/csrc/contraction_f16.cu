// contraction_f16.cu -- batched FP16 contractions on the 5th-generation tensor cores with f32
// accumulation, for the attention products of a transformer encoder block (BERT-base shape:
// scores = Q K^T / sqrt(64), O = P V, per batch and head):
//   C[bb][m][n] = alpha * sum_k A[bb][m][k] * B[bb][n][k],   bb = b * heads + h
// Operands are read through 4-D tensor maps {k, row, head, batch} with arbitrary row / head /
// batch strides, so Q, K and V are read in place from the fused QKV projection output
// ([B, S, 3 x heads, 64]) and C is written through (row, head, batch) strides (e.g. straight
// into [B, S, heads x 64]).  Pipeline as the INT8 kernel: warp 0 TMA producer, warp 1 issues
// tcgen05.mma.kind::f16 (M = 128, N = BN, K = 16), warps 2-9 epilogue from a double-buffered
// TMEM accumulator; every wait is bounded.
#include <cuda_fp16.h>

#include <mutex>

#include "lsc_internal.h"
#include "sm100.cuh"

namespace lsc {
namespace {

struct F16Params {
  int32_t m, n, k;           // per-batch GEMM
  int32_t heads, batches;    // bb = b * heads + h
  int32_t a_head0, b_head0;  // head coordinate of head 0 in the A / B maps
  float alpha;
  void* out;
  int32_t out_f16;
  int64_t cs_row, cs_head, cs_batch;  // output element strides
  int32_t vec_ok;
  uint32_t* err;
};

template <int BN_>
struct F16Cfg {
  static constexpr int BM = 128;
  static constexpr int BN = BN_;
  static constexpr int BK = 64;  // f16 elements of K per stage (128 bytes)
  static constexpr int A_BYTES = BM * 128;
  static constexpr int B_BYTES = BN * 128;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (196608 / STAGE_BYTES) < 8 ? (196608 / STAGE_BYTES) : 8;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int EPI_WARPS = 8;
  static constexpr int THREADS = 64 + 32 * EPI_WARPS;
  static constexpr int COLS_PER_EPI_WARP = BN / 2;
  static constexpr int BAR_BYTES = 256;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + BAR_BYTES;
  static constexpr uint32_t IDESC = idesc_f16(BM, BN);
  static_assert(SMEM_BYTES <= 232448, "shared memory budget");
  static_assert((2 * STAGES + 5) * 8 + 8 <= BAR_BYTES, "barrier area");
};

__device__ __forceinline__ void store_chunk(const F16Params& p, const uint32_t (&r)[32], int64_t base, int col0) {
  const bool full = col0 + 32 <= p.n;
  float v[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __fmul_rn(__uint_as_float(r[j]), p.alpha);
  if (p.out_f16) {
    __half* o = static_cast<__half*>(p.out) + base;
    if (full && p.vec_ok) {
      uint32_t w[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const __half2 h = __floats2half2_rn(v[2 * j], v[2 * j + 1]);
        w[j] = *reinterpret_cast<const uint32_t*>(&h);
      }
      uint4* d = reinterpret_cast<uint4*>(o);
#pragma unroll
      for (int j = 0; j < 4; ++j) d[j] = make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (col0 + j < p.n) o[j] = __float2half_rn(v[j]);
    }
  } else {
    float* o = static_cast<float*>(p.out) + base;
    if (full && p.vec_ok) {
      float4* d = reinterpret_cast<float4*>(o);
#pragma unroll
      for (int j = 0; j < 8; ++j) d[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (col0 + j < p.n) o[j] = v[j];
    }
  }
}

template <int BN>
__global__ void __launch_bounds__(F16Cfg<BN>::THREADS, 1)
    contraction_f16_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                           const F16Params p) {
  using C = F16Cfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + C::STAGES * C::A_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::STAGES * C::STAGE_BYTES);
  uint64_t* full = bars;
  uint64_t* empty = bars + C::STAGES;
  uint64_t* tfull = bars + 2 * C::STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile uint32_t* abort_flag = tmem_slot + 1;

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
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int m_tiles = (p.m + C::BM - 1) / C::BM;
  const int n_tiles = (p.n + C::BN - 1) / C::BN;
  const int per_batch = m_tiles * n_tiles;
  const int num_tiles = per_batch * p.batches;
  const int kblocks = (p.k + C::BK - 1) / C::BK;

  if (warp == 0) {
    if (lane == 0) {
      uint32_t stage = 0, phase = 0;
      int issued = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int bb = tile / per_batch, t = tile - bb * per_batch;
        const int mb = t % m_tiles, nb = t / m_tiles;
        const int b = bb / p.heads, h = bb - b * p.heads;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, p.err)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
          tma_load_4d(&tmA, &full[stage], sA + stage * C::A_BYTES, kb * C::BK, mb * C::BM, p.a_head0 + h, b);
          tma_load_4d(&tmB, &full[stage], sB + stage * C::B_BYTES, kb * C::BK, nb * C::BN, p.b_head0 + h, b);
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
          mbar_wait(&full[idx % C::STAGES], static_cast<uint32_t>((idx / C::STAGES) & 1), &no_abort, p.err);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      uint32_t stage = 0, phase = 0;
      int local = 0;
      bool ok = true;
      bool any_mma = false;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++local) {
        const int buf = local & 1;
        if (!mbar_wait(&tempty[buf], static_cast<uint32_t>((local >> 1) & 1) ^ 1u, abort_flag, p.err)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * C::BN);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, p.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + stage * C::A_BYTES);
          const uint32_t b0 = smem_u32(sB + stage * C::B_BYTES);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)  // 4 x K=16 per 128-byte stage
            mma_f16(d_tmem, smem_desc_sw128_kmajor(a0 + kk * 32), smem_desc_sw128_kmajor(b0 + kk * 32), C::IDESC,
                    (kb | kk) != 0 ? 1u : 0u);
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
    int local = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      const int bb = tile / per_batch, t = tile - bb * per_batch;
      const int mb = t % m_tiles, nb = t / m_tiles;
      const int b = bb / p.heads, h = bb - b * p.heads;
      const int buf = local & 1;
      if (!mbar_wait(&tfull[buf], static_cast<uint32_t>((local >> 1) & 1), abort_flag, p.err)) break;
      tc_fence_after();
      const int row = mb * C::BM + quarter * 32 + lane;
      const int64_t rbase = b * p.cs_batch + h * p.cs_head + static_cast<int64_t>(row) * p.cs_row;
      constexpr int CHUNKS = C::COLS_PER_EPI_WARP / 32;
#pragma unroll 1
      for (int c = 0; c < CHUNKS; ++c) {
        const int tcol = half * C::COLS_PER_EPI_WARP + c * 32;
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                               static_cast<uint32_t>(buf * C::BN + tcol),
                           r);
        tmem_ld_wait();
        if (c == CHUNKS - 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tempty[buf]);
        }
        const int col0 = nb * C::BN + tcol;
        if (row < p.m && col0 < p.n) store_chunk(p, r, rbase + col0, col0);
      }
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

template <int BN>
lsc_status launch_f16(const CUtensorMap& ta, const CUtensorMap& tb, const F16Params& p, int sm_count,
                      cudaStream_t stream) {
  using C = F16Cfg<BN>;
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [] {
    attr_err = cudaFuncSetAttribute(contraction_f16_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    C::SMEM_BYTES);
  });
  if (attr_err != cudaSuccess) return cuda_error(attr_err, "cudaFuncSetAttribute(contraction_f16)");
  const int64_t tiles =
      static_cast<int64_t>((p.m + C::BM - 1) / C::BM) * ((p.n + C::BN - 1) / C::BN) * p.batches;
  const int grid = static_cast<int>(tiles < sm_count ? tiles : sm_count);
  contraction_f16_kernel<BN><<<grid, C::THREADS, C::SMEM_BYTES, stream>>>(ta, tb, p);
  LSC_CUDA_TRY(cudaGetLastError());
  return LSC_SUCCESS;
}

// Operand map {k, row, head, batch}: element (b, head, row, k) at base + b*sb + head*sh + row*sr + k.
lsc_status operand_map(CUtensorMap* map, const void* base, int64_t rows, int64_t k, int64_t heads_extent,
                       int64_t batches, int64_t sr, int64_t sh, int64_t sb, uint32_t box_rows) {
  if (((sr | sh | sb) * 2) % 16 != 0)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "gemm_f16: operand strides must be multiples of 8 elements");
  const uint64_t dims[4] = {static_cast<uint64_t>(k), static_cast<uint64_t>(rows), static_cast<uint64_t>(heads_extent),
                            static_cast<uint64_t>(batches)};
  const uint64_t strides[3] = {static_cast<uint64_t>(sr * 2), static_cast<uint64_t>(sh * 2),
                               static_cast<uint64_t>(sb * 2)};
  const uint32_t box[4] = {64, box_rows, 1, 1};
  const uint32_t ones[4] = {1, 1, 1, 1};
  return encode_tmap_4d(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, base, dims, strides, box, ones, CU_TENSOR_MAP_SWIZZLE_128B);
}

// [B][H][R][Cc] <- transpose of the (h + h0) head slot of x, element (b, h, r, c) at
// x + b*xb + (h + h0)*xh + r*xr + c, for the B operand of O = P V (V^T, K-major).
__global__ void transpose_heads_f16_kernel(const __half* __restrict__ x, __half* __restrict__ y, int64_t xb,
                                           int64_t xh, int64_t xr, int h0, int heads, int rows, int cols) {
  __shared__ __half tile[32][33];
  const int bh = blockIdx.z;
  const int b = bh / heads, h = bh - b * heads;
  const __half* src = x + b * xb + (h + h0) * xh;
  __half* dst = y + static_cast<int64_t>(bh) * rows * cols;
  const int r0 = blockIdx.y * 32, c0 = blockIdx.x * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int r = r0 + i, c = c0 + threadIdx.x;
    if (r < rows && c < cols) tile[i][threadIdx.x] = src[static_cast<int64_t>(r) * xr + c];
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int c = c0 + i, r = r0 + threadIdx.x;
    if (r < rows && c < cols) dst[static_cast<int64_t>(c) * rows + r] = tile[threadIdx.x][i];
  }
}

}  // namespace

lsc_status launch_gemm_f16_batched(const void* a, int64_t as_row, int64_t as_head, int64_t as_batch, int64_t a_head0,
                                   const void* bm, int64_t bs_row, int64_t bs_head, int64_t bs_batch, int64_t b_head0,
                                   int64_t batch, int64_t heads, int64_t m, int64_t n, int64_t k, float alpha,
                                   void* c, int32_t c_dtype, int64_t cs_row, int64_t cs_head, int64_t cs_batch,
                                   cudaStream_t stream) {
  if (batch < 0 || heads <= 0 || m < 0 || n < 0 || k < 0 || a_head0 < 0 || b_head0 < 0)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "gemm_f16: bad sizes");
  if (batch == 0 || m == 0 || n == 0) return LSC_SUCCESS;
  if (k == 0 || k % 8 != 0) return set_error(LSC_ERROR_INVALID_ARGUMENT, "gemm_f16: K must be a positive multiple of 8");
  if (!a || !bm || !c) return set_error(LSC_ERROR_INVALID_ARGUMENT, "gemm_f16: null pointer");
  if (c_dtype != LSC_DTYPE_F16 && c_dtype != LSC_DTYPE_F32)
    return set_error(LSC_ERROR_UNSUPPORTED_DATATYPE, "gemm_f16: output must be f16 or f32");
  if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(bm)) & 15)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "gemm_f16: operands must be 16-byte aligned");
  if (m > INT32_MAX / 2 || n > INT32_MAX / 2 || k > INT32_MAX / 2 || batch * heads > INT32_MAX / 4)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "gemm_f16: size too large");
  DeviceState* ds = current_device_state();
  if (!ds) return LSC_ERROR_DEVICE_ERROR;
  if (ds->cc_major != 10) return set_error(LSC_ERROR_BACKEND_NOT_AVAILABLE, "gemm_f16: needs an sm_100 device");
  const int bn = n <= 64 ? 64 : (n <= 128 || n % 256 != 0 ? 128 : 256);
  CUtensorMap ta, tb;
  lsc_status st = operand_map(&ta, a, m, k, a_head0 + heads, batch, as_row, as_head, as_batch, 128);
  if (st) return st;
  if ((st = operand_map(&tb, bm, n, k, b_head0 + heads, batch, bs_row, bs_head, bs_batch, static_cast<uint32_t>(bn))))
    return st;
  F16Params p{};
  p.m = static_cast<int32_t>(m);
  p.n = static_cast<int32_t>(n);
  p.k = static_cast<int32_t>(k);
  p.heads = static_cast<int32_t>(heads);
  p.batches = static_cast<int32_t>(batch * heads);
  p.a_head0 = static_cast<int32_t>(a_head0);
  p.b_head0 = static_cast<int32_t>(b_head0);
  p.alpha = alpha;
  p.out = c;
  p.out_f16 = c_dtype == LSC_DTYPE_F16 ? 1 : 0;
  p.cs_row = cs_row;
  p.cs_head = cs_head;
  p.cs_batch = cs_batch;
  const int esz = p.out_f16 ? 2 : 4;
  p.vec_ok = ((reinterpret_cast<uintptr_t>(c) & 15) == 0 && ((cs_row | cs_head | cs_batch) * esz) % 16 == 0) ? 1 : 0;
  p.err = ds->err_word;
  switch (bn) {
    case 64: return launch_f16<64>(ta, tb, p, ds->sm_count, stream);
    case 128: return launch_f16<128>(ta, tb, p, ds->sm_count, stream);
    default: return launch_f16<256>(ta, tb, p, ds->sm_count, stream);
  }
}

lsc_status launch_transpose_heads_f16(const void* x, void* y, int64_t xb, int64_t xh, int64_t xr, int64_t h0,
                                      int64_t batch, int64_t heads, int64_t rows, int64_t cols, cudaStream_t stream) {
  if (batch < 0 || heads <= 0 || rows < 0 || cols < 0 || h0 < 0)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "transpose_heads_f16: bad sizes");
  if (batch == 0 || rows == 0 || cols == 0) return LSC_SUCCESS;
  if (batch * heads > 65535 || rows > INT32_MAX / 2 || cols > INT32_MAX / 2)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "transpose_heads_f16: too large");
  const dim3 grid(static_cast<unsigned>((cols + 31) / 32), static_cast<unsigned>((rows + 31) / 32),
                  static_cast<unsigned>(batch * heads));
  transpose_heads_f16_kernel<<<grid, dim3(32, 8), 0, stream>>>(static_cast<const __half*>(x), static_cast<__half*>(y),
                                                               xb, xh, xr, static_cast<int>(h0),
                                                               static_cast<int>(heads), static_cast<int>(rows),
                                                               static_cast<int>(cols));
  LSC_CUDA_TRY(cudaGetLastError());
  return LSC_SUCCESS;
}

}  // namespace lsc

extern "C" lsc_status lsc_gemm_f16_batched(const void* a, int64_t as_row, int64_t as_head, int64_t as_batch,
                                           int64_t a_head0, const void* b, int64_t bs_row, int64_t bs_head,
                                           int64_t bs_batch, int64_t b_head0, int64_t batch, int64_t heads,
                                           int64_t m, int64_t n, int64_t k, float alpha, void* c, int32_t c_dtype,
                                           int64_t cs_row, int64_t cs_head, int64_t cs_batch, lsc_stream stream) {
  return lsc::launch_gemm_f16_batched(a, as_row, as_head, as_batch, a_head0, b, bs_row, bs_head, bs_batch, b_head0,
                                      batch, heads, m, n, k, alpha, c, c_dtype, cs_row, cs_head, cs_batch,
                                      static_cast<cudaStream_t>(stream));
}

extern "C" lsc_status lsc_transpose_heads_f16(const void* x, void* y, int64_t x_batch_stride,
                                              int64_t x_head_stride, int64_t x_row_stride, int64_t head0,
                                              int64_t batch, int64_t heads, int64_t rows, int64_t cols,
                                              lsc_stream stream) {
  return lsc::launch_transpose_heads_f16(x, y, x_batch_stride, x_head_stride, x_row_stride, head0, batch, heads, rows,
                                         cols, static_cast<cudaStream_t>(stream));
}
