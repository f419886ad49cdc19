// attention_f16.cu -- fused multi-head attention of a transformer encoder block (BERT-base
// shape: head dim 64, sequence up to 384) on the 5th-generation tensor cores:
//   O[b, q, h, :] = sum_k P[q, k] V[b, k, h, :],   P = f16(softmax(f16(alpha * Q K^T)))
// with the rounding points of the unfused path (scores stored as f16, probabilities as f16,
// products accumulated in f32), so it computes what the FP16 GEMM, the Softmax operator and
// the FP16 GEMM compute one after another, without the [batch, heads, seq, seq] round trips
// through HBM.  The reference engine declares MultiHeadAttention (core/ir/operator.rs:54-58,
// core/operator/attention.rs) but its CPU backend computes no attention; the softmax follows
// operator/softmax.rs:106-146 (max, exp(x - max), times 1 / sum).
//
// One CTA per SM walks a contiguous range of (batch, head, 128-query tile) units:
//   warp 0      TMA producer: K and V ([seq, 64] each, straight from the QKV projection) once
//               per (batch, head), Q ([128, 64]) per unit;
//   warp 1      MMA issuer: S = Q K^T into TMEM columns [0, seq) (M = 128, N <= 256, K = 16
//               steps), then O = P V into columns [384, 448) with V read MN-major (its rows
//               are keys, the contraction index, with the 64 head dims contiguous);
//   warps 2-17  softmax and epilogue: warp (quarter, part) owns 32 query rows (its TMEM lane
//               quarter) and seq/4 key columns, in chunks of 32.  Pass 1 rounds the chunk's
//               scores to f16, takes their max m_c and writes e = exp(x - m_c) (2^((x - m_c)
//               log2 e) on the MUFU unit) back to TMEM with the chunk sum; the row max m and
//               sum (chunk sums rescaled by exp(m_c - m)) are combined over the four parts
//               through shared memory; pass 2 writes P = f16(e exp(m_c - m) / sum) to shared
//               memory in the 128-byte-swizzled K-major layout the P V MMA reads; O is written
//               as f32 and/or quantized to int8 (the Quantize operator's arithmetic).
// Every wait is bounded (a timeout flags the device error word and ends the CTA's work).
#include <cuda_fp16.h>

#include <mutex>

#include "epilogue.cuh"
#include "lsc_internal.h"
#include "sm100.cuh"

namespace lsc {
namespace {

constexpr int kHeadDim = 64;
constexpr int kMaxSeq = 384;
constexpr int kSoftWarps = 16;
constexpr int kAttnThreads = 64 + 32 * kSoftWarps;
constexpr int kKBytes = kMaxSeq * 128;      // K rows, 128 bytes each
constexpr int kVBytes = kMaxSeq * 128;      // V rows (keys), 128 bytes each
constexpr int kQBytes = 128 * 128;
constexpr int kPBytes = kMaxSeq * 256;      // seq/64 chunks of [128 rows x 128 B]
constexpr int kRedBytes = 2 * 4 * 128 * 4;  // row max and row sum per part
constexpr int kBarBytes = 128;  // 9 mbarriers, the TMEM address and the abort flag
constexpr int kAttnSmem = kKBytes + kVBytes + kQBytes + kPBytes + kRedBytes + kBarBytes + 1024;
constexpr uint32_t kOCol = 384;             // TMEM column of O
constexpr float kLog2e = 1.4426950408889634f;
static_assert(kAttnSmem <= 232448, "shared memory budget");

struct AttnParams {
  int32_t batch, seq, heads;
  float alpha;
  float* out_f32;   // [batch * seq, heads * 64] or null
  int8_t* out_i8;   // same layout, or null
  float s_out, inv_s_out;
  int32_t rounding;
  uint32_t* err;
};

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// {lo, hi} rounded to f16 and packed (lo in the low half)
__device__ __forceinline__ uint32_t f16x2_rn(float lo, float hi) {
  uint32_t d;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}
// lane-wise max of two f16 pairs (a NaN operand yields the other one, as f32::max)
__device__ __forceinline__ uint32_t hmax2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("max.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
// the two halves of an f16 pair plus c, in f32 (mixed-precision add: one rounding, exact
// when c is an f16 value or zero)
__device__ __forceinline__ void f16x2_to_f32(uint32_t h2, float c, float& lo, float& hi) {
  asm("{\n .reg .b16 l, h;\n mov.b32 {l, h}, %2;\n add.rn.f32.f16 %0, l, %3;\n add.rn.f32.f16 %1, h, %3;\n}"
      : "=f"(lo), "=f"(hi)
      : "r"(h2), "f"(c));
}

// unit u of [0, batch * heads * qtiles): (batch * heads + head, query tile)
struct Unit {
  int bh, qt;
};
__device__ __forceinline__ Unit unit_of(int u, int qtiles) { return {u / qtiles, u % qtiles}; }

__global__ void __launch_bounds__(kAttnThreads, 1)
    attention_f16_kernel(const __grid_constant__ CUtensorMap tmQKV, const AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sK = smem;
  uint8_t* sV = sK + kKBytes;
  uint8_t* sQ = sV + kVBytes;
  uint8_t* sP = sQ + kQBytes;
  float* red_max = reinterpret_cast<float*>(sP + kPBytes);
  float* red_sum = red_max + 4 * 128;
  uint64_t* bars = reinterpret_cast<uint64_t*>(red_sum + 4 * 128);
  uint64_t* kv_full = bars + 0;
  uint64_t* kv_empty = bars + 1;
  uint64_t* q_full = bars + 2;
  uint64_t* q_empty = bars + 3;
  uint64_t* s_full = bars + 4;
  uint64_t* p_full = bars + 5;
  uint64_t* o_full = bars + 6;
  uint64_t* drain = bars + 7;
  uint64_t* rmax_bar = bars + 8;  // the 16 softmax warps' row maxima and sums are in red_*
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 9);
  volatile uint32_t* abort_flag = tmem_slot + 1;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int seq = p.seq;
  const int qtiles = seq / 128;
  const int units = p.batch * p.heads * qtiles;
  const int u_begin = static_cast<int>((static_cast<int64_t>(blockIdx.x) * units) / gridDim.x);
  const int u_end = static_cast<int>((static_cast<int64_t>(blockIdx.x + 1) * units) / gridDim.x);

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    mbar_init(kv_empty, 1);
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    mbar_init(s_full, 1);
    mbar_init(p_full, kSoftWarps);
    mbar_init(o_full, 1);
    mbar_init(drain, 1);
    mbar_init(rmax_bar, kSoftWarps);
    *abort_flag = 0u;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmQKV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------------ TMA producer
      uint32_t kv_ph = 0, q_ph = 0;
      int reloads = 0, q_loads = 0;
      int cur_bh = -1;
      bool ok = true;
      for (int u = u_begin; u < u_end && ok; ++u) {
        const Unit un = unit_of(u, qtiles);
        const int b = un.bh / p.heads, h = un.bh - b * p.heads;
        if (un.bh != cur_bh) {
          if (cur_bh >= 0 && !(ok = mbar_wait(kv_empty, kv_ph, abort_flag, p.err))) break;
          if (cur_bh >= 0) kv_ph ^= 1u;
          mbar_arrive_expect_tx(kv_full, static_cast<uint32_t>(2 * seq * 128));
          for (int i = 0; i < seq / 128; ++i) {
            tma_load_4d(&tmQKV, kv_full, sK + i * 16384, 0, i * 128, p.heads + h, b);
            tma_load_4d(&tmQKV, kv_full, sV + i * 16384, 0, i * 128, 2 * p.heads + h, b);
          }
          ++reloads;
          cur_bh = un.bh;
        }
        if (!(ok = mbar_wait(q_empty, q_ph ^ 1u, abort_flag, p.err))) break;
        q_ph ^= 1u;
        mbar_arrive_expect_tx(q_full, kQBytes);
        tma_load_4d(&tmQKV, q_full, sQ, 0, un.qt * 128, h, b);
        ++q_loads;
      }
      if (!ok) {
        // let the copies in flight land before the CTA exits (their barriers complete)
        volatile uint32_t no_abort = 0;
        if (reloads > 0) mbar_wait(kv_full, static_cast<uint32_t>((reloads - 1) & 1), &no_abort, p.err);
        if (q_loads > 0) mbar_wait(q_full, static_cast<uint32_t>((q_loads - 1) & 1), &no_abort, p.err);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------------ MMA issuer
      uint32_t kv_ph = 0, q_ph = 0, p_ph = 0;
      int cur_bh = -1;
      bool ok = true, any_mma = false;
      for (int u = u_begin; u < u_end && ok; ++u) {
        const Unit un = unit_of(u, qtiles);
        if (un.bh != cur_bh) {
          if (!(ok = mbar_wait(kv_full, kv_ph, abort_flag, p.err))) break;
          kv_ph ^= 1u;
          cur_bh = un.bh;
        }
        if (!(ok = mbar_wait(q_full, q_ph, abort_flag, p.err))) break;
        q_ph ^= 1u;
        tc_fence_after();
        // S = Q K^T: N blocks of up to 256 keys
        const uint32_t q0 = smem_u32(sQ);
        for (int n0 = 0; n0 < seq; n0 += 256) {
          const int nb = seq - n0 < 256 ? seq - n0 : 256;
          const uint32_t idesc = idesc_f16(128, static_cast<uint32_t>(nb));
          const uint32_t k0 = smem_u32(sK + n0 * 128);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_f16(tmem_base + static_cast<uint32_t>(n0), smem_desc_sw128_kmajor(q0 + kk * 32),
                    smem_desc_sw128_kmajor(k0 + kk * 32), idesc, kk != 0 ? 1u : 0u);
        }
        any_mma = true;
        mma_commit(q_empty);
        mma_commit(s_full);
        if (!(ok = mbar_wait(p_full, p_ph, abort_flag, p.err))) break;
        p_ph ^= 1u;
        tc_fence_after();
        // O = P V: K = seq in steps of 16 keys; P K-major (64-key chunks of 128-byte rows),
        // V MN-major (16 key rows = two 8-row swizzle atoms = 2048 bytes per step)
        constexpr uint32_t idesc_o = idesc_f16_bmn(128, kHeadDim);
        for (int c = 0; c < seq / 64; ++c) {
          const uint32_t pa = smem_u32(sP + c * 16384);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_f16(tmem_base + kOCol, smem_desc_sw128_kmajor(pa + kk * 32),
                    smem_desc_sw128_mnmajor(smem_u32(sV + (4 * c + kk) * 2048), 0), idesc_o, (c | kk) != 0 ? 1u : 0u);
        }
        mma_commit(o_full);
        // K / V are reloaded before the next unit of another (batch, head)
        if (u + 1 < u_end && unit_of(u + 1, qtiles).bh != cur_bh) mma_commit(kv_empty);
      }
      if (!ok && any_mma) {
        volatile uint32_t no_abort = 0;
        mma_commit(drain);
        mbar_wait(drain, 0u, &no_abort, p.err);
      }
    }
  } else {
    // -------------------------------------------------------------------- softmax + epilogue
    const int sw = warp - 2;
    const int quarter = warp & 3;
    const int part = sw >> 2;
    const int row = quarter * 32 + lane;                 // query row within the tile (TMEM lane)
    const int ncols = seq / 4;                           // key columns of this warp
    const int col0 = part * ncols;
    const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
    uint32_t s_ph = 0, o_ph = 0, r_ph = 0;
    for (int u = u_begin; u < u_end; ++u) {
      const Unit un = unit_of(u, qtiles);
      const int b = un.bh / p.heads, h = un.bh - b * p.heads;
      if (!mbar_wait(s_full, s_ph, abort_flag, p.err)) break;
      s_ph ^= 1u;
      tc_fence_after();
      // pass 1, per 32-column chunk c: the f16 scores, their max m_c, e = 2^((x - m_c) log2 e)
      // back into TMEM and the chunk sum s_c.  A chunk whose scores are all -inf uses 0 as
      // its reference (its e are 0).
      float mc[3], sc[3];
      float m_thr = -INFINITY;
      const int nch = ncols >> 5;
#pragma unroll
      for (int c = 0; c < 3; ++c) {
        mc[c] = 0.0f;
        sc[c] = 0.0f;
        if (c >= nch) continue;
        uint32_t r[32];
        tmem_ld_32x32b_x32(t_row + static_cast<uint32_t>(col0 + 32 * c), r);
        tmem_ld_wait();
        uint32_t hx[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          float a, bb;
          f2unpack(f2mul(f2pack(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1])), f2pack(p.alpha, p.alpha)),
                   a, bb);
          hx[j] = f16x2_rn(a, bb);
        }
        uint32_t hm = hx[0];
#pragma unroll
        for (int j = 1; j < 16; ++j) hm = hmax2(hm, hx[j]);
        float m0, m1;
        f16x2_to_f32(hm, 0.0f, m0, m1);
        float m = fmaxf(m0, m1);
        const float ref = m == -INFINITY ? 0.0f : m;
        float s_c = 0.0f;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          float x0, x1;
          f16x2_to_f32(hx[j], -ref, x0, x1);  // x - ref, exact
          f2unpack(f2mul(f2pack(x0, x1), f2pack(kLog2e, kLog2e)), x0, x1);
          const float e0 = ex2_approx(x0), e1 = ex2_approx(x1);
          s_c = __fadd_rn(s_c, __fadd_rn(e0, e1));
          r[2 * j] = __float_as_uint(e0);
          r[2 * j + 1] = __float_as_uint(e1);
        }
        tmem_st_32x32b_x32(t_row + static_cast<uint32_t>(col0 + 32 * c), r);
        mc[c] = ref;
        sc[c] = s_c;
        m_thr = fmaxf(m_thr, m);
      }
      tmem_st_wait();
      // this thread's share of the row: max and sum rescaled to it; combined over the parts
      const float ref_thr = m_thr == -INFINITY ? 0.0f : m_thr;
      float s_thr = 0.0f;
#pragma unroll
      for (int c = 0; c < 3; ++c)
        if (c < nch) s_thr = __fadd_rn(s_thr, __fmul_rn(sc[c], ex2_approx((mc[c] - ref_thr) * kLog2e)));
      red_max[part * 128 + row] = ref_thr;
      red_sum[part * 128 + row] = s_thr;
      __syncwarp();
      if (lane == 0) mbar_arrive(rmax_bar);
      if (!mbar_wait(rmax_bar, r_ph, abort_flag, p.err)) break;
      r_ph ^= 1u;
      float m_row = red_max[row];
#pragma unroll
      for (int q = 1; q < 4; ++q) m_row = fmaxf(m_row, red_max[q * 128 + row]);
      float sum = 0.0f;
#pragma unroll
      for (int q = 0; q < 4; ++q)
        sum = __fadd_rn(sum, __fmul_rn(red_sum[q * 128 + row], ex2_approx((red_max[q * 128 + row] - m_row) * kLog2e)));
      const bool normal = sum > 0.0f && sum < INFINITY;
      const float inv = normal ? __fdiv_rn(1.0f, sum) : 0.0f;
      // pass 2: P = f16(e * 2^((m_c - m_row) log2 e) / sum) into the swizzled K-major A tile of O = P V
#pragma unroll
      for (int c = 0; c < 3; ++c) {
        if (c >= nch) continue;
        uint32_t r[32];
        tmem_ld_32x32b_x32(t_row + static_cast<uint32_t>(col0 + 32 * c), r);
        tmem_ld_wait();
        const float f = __fmul_rn(ex2_approx((mc[c] - m_row) * kLog2e), inv);
        uint32_t w[16];
        if (normal) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            float a, bb;
            f2unpack(f2mul(f2pack(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1])), f2pack(f, f)), a, bb);
            w[j] = f16x2_rn(a, bb);
          }
        } else {
          // no finite positive normaliser (an infinite or NaN score in the row): the row's
          // probabilities are NaN, so its output is NaN
#pragma unroll
          for (int j = 0; j < 16; ++j) w[j] = 0x7E007E00u;
        }
        const int key = col0 + 32 * c;
        uint8_t* chunk = sP + (key >> 6) * 16384 + row * 128;
        const int g0 = (key & 63) >> 3;
#pragma unroll
        for (int i = 0; i < 4; ++i)
          *reinterpret_cast<uint4*>(chunk + (((g0 + i) ^ (row & 7)) << 4)) =
              make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
      // epilogue: O rows of this quarter, 16 head-dim columns per part
      if (!mbar_wait(o_full, o_ph, abort_flag, p.err)) break;
      o_ph ^= 1u;
      tc_fence_after();
      uint32_t r[16];
      tmem_ld_32x32b_x16(t_row + kOCol + static_cast<uint32_t>(part * 16), r);
      tmem_ld_wait();
      const int64_t token = static_cast<int64_t>(b) * seq + un.qt * 128 + row;
      const int64_t base = token * (p.heads * kHeadDim) + h * kHeadDim + part * 16;
      float y[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) y[j] = __uint_as_float(r[j]);
      if (p.out_f32) {
#pragma unroll
        for (int v = 0; v < 2; ++v) {
          uint32_t o[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) o[j] = r[8 * v + j];
          st_global_v8(p.out_f32 + base + 8 * v, o);
        }
      }
      if (p.out_i8) {
        uint32_t pk[4];
        requant_pack<16>(y, p.s_out, p.inv_s_out, false, p.rounding, pk);
        *reinterpret_cast<uint4*>(p.out_i8 + base) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

}  // namespace

lsc_status launch_attention_f16(const void* qkv, int64_t batch, int64_t seq, int64_t heads, float alpha,
                                float* out_f32, int8_t* out_i8, float s_out, int rounding, cudaStream_t stream) {
  if (batch < 0 || heads <= 0 || seq <= 0) return set_error(LSC_ERROR_INVALID_ARGUMENT, "attention_f16: bad sizes");
  if (seq % 128 != 0 || seq > kMaxSeq)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "attention_f16: seq must be a multiple of 128, at most %d", kMaxSeq);
  if (batch == 0) return LSC_SUCCESS;
  if (!qkv || (!out_f32 && !out_i8)) return set_error(LSC_ERROR_INVALID_ARGUMENT, "attention_f16: null pointer");
  if ((reinterpret_cast<uintptr_t>(qkv) | reinterpret_cast<uintptr_t>(out_i8)) & 15)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "attention_f16: buffers must be 16-byte aligned");
  if (reinterpret_cast<uintptr_t>(out_f32) & 31)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "attention_f16: the f32 output must be 32-byte aligned");
  if (out_i8 && !(s_out > 0.0f)) return set_error(LSC_ERROR_INVALID_ARGUMENT, "attention_f16: int8 output needs a scale > 0");
  if (batch * heads * seq > INT32_MAX / 4 || batch * heads > 65535)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "attention_f16: too large");
  DeviceState* ds = current_device_state();
  if (!ds) return LSC_ERROR_DEVICE_ERROR;
  if (ds->cc_major != 10) return set_error(LSC_ERROR_BACKEND_NOT_AVAILABLE, "attention_f16: needs an sm_100 device");
  // {head dim, token, head slot (Q 0..H-1, K H..2H-1, V 2H..3H-1), batch} over [batch, seq, 3, heads, 64]
  const int64_t row = 3 * heads * kHeadDim;
  CUtensorMap tm;
  const uint64_t dims[4] = {kHeadDim, static_cast<uint64_t>(seq), static_cast<uint64_t>(3 * heads),
                            static_cast<uint64_t>(batch)};
  const uint64_t strides[3] = {static_cast<uint64_t>(row * 2), kHeadDim * 2, static_cast<uint64_t>(seq * row * 2)};
  const uint32_t box[4] = {64, 128, 1, 1};
  const uint32_t ones[4] = {1, 1, 1, 1};
  lsc_status st = encode_tmap_4d(&tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, qkv, dims, strides, box, ones,
                                 CU_TENSOR_MAP_SWIZZLE_128B);
  if (st) return st;
  AttnParams p{};
  p.batch = static_cast<int32_t>(batch);
  p.seq = static_cast<int32_t>(seq);
  p.heads = static_cast<int32_t>(heads);
  p.alpha = alpha;
  p.out_f32 = out_f32;
  p.out_i8 = out_i8;
  p.s_out = s_out;
  p.inv_s_out = out_i8 ? reciprocal_or_zero(s_out) : 0.0f;
  p.rounding = rounding;
  p.err = ds->err_word;
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [] {
    attr_err = cudaFuncSetAttribute(attention_f16_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kAttnSmem);
  });
  if (attr_err != cudaSuccess) return cuda_error(attr_err, "cudaFuncSetAttribute(attention_f16)");
  const int64_t units = batch * heads * (seq / 128);
  const int grid = static_cast<int>(units < ds->sm_count ? units : ds->sm_count);
  attention_f16_kernel<<<grid, kAttnThreads, kAttnSmem, stream>>>(tm, p);
  LSC_CUDA_TRY(cudaGetLastError());
  return LSC_SUCCESS;
}

}  // namespace lsc

extern "C" lsc_status lsc_attention_f16(const void* qkv, int64_t batch, int64_t seq, int64_t heads, float alpha,
                                        float* out_f32, int8_t* out_i8, float s_out, int32_t rounding,
                                        lsc_stream stream) {
  return lsc::launch_attention_f16(qkv, batch, seq, heads, alpha, out_f32, out_i8, s_out, rounding,
                                   static_cast<cudaStream_t>(stream));
}
