// contraction_i8.cu -- INT8 x INT8 -> INT32 contractions on the 5th-generation tensor cores
// with the requantize / dequantize epilogue fused in:
//   * GEMM  C[M,N] = A[M,K] W[N,K]^T      replaces quantized_gemm_int8 + dequantize +
//                                         quantize_sym (lightship-core/src/cpu/quantized_ops.rs:13-48)
//   * NHWC convolution as an implicit GEMM (M = N*OH*OW output pixels, K = KH*KW*C) --
//     the INT8 counterpart of Conv2d::forward's im2col + GEMM
//     (lightship-core/src/operator/convolution.rs:90-267) with the column matrix never
//     materialised: the TMA engine gathers it in im2col mode straight into shared memory.
//
// Design (one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer: the A tile (128 rows x 128 B of K) -- a 2-D tile for GEMM, or
//               128/ACB im2col loads of ACB channels each for convolution -- and the W tile
//               (BN rows x 128 B), into a STAGES-deep shared-memory ring (full/empty mbarriers).
//   warp 1      MMA issuer: one thread issues tcgen05.mma.kind::i8 (M=128, N=BN, K=32) into a
//               double-buffered s32 accumulator in TMEM (2 x BN columns) and commits each
//               stage back to the producer and each finished tile to the epilogue.
//   warps 2-17  epilogue: tcgen05.ld of the accumulator (warp w reads TMEM lanes
//               32*(w%4)..+31 and a quarter of the tile's columns, 16 at a time), bias,
//               per-channel scale, activation, requantize, vectorised global stores.  Four
//               warps per SM sub-partition keep the TMEM loads and the requantization's
//               dependent chains overlapped.  The accumulator buffer is released right after
//               its last TMEM read so the next tile's MMAs overlap this tile's epilogue math.
#include <math.h>
#include <stdlib.h>
#include <stdio.h>

#include <mutex>

#include <cuda_fp16.h>

#include "epilogue.cuh"
#include "lsc_internal.h"
#include "sm100.cuh"

namespace lsc {
namespace {

struct I8Params {
  int32_t m, n, k;  // GEMM view: rows, output channels, K bytes
  const int32_t* bias;
  const float* scale;
  float s_out;
  float inv_s_out;  // RN(1 / s_out) when s_out and its reciprocal are normal floats, else 0
  int32_t rounding;
  int8_t* out_i8;
  float* out_f32;
  int32_t* out_i32;
  __half* out_f16;        // optional f16 copy of the f32 output (after the activation)
  const float* res_f32;   // optional f32 residual [M, ldo] added before the activation
  int64_t ldo;
  int32_t vec_ok;  // 16-byte vector stores are legal for full column chunks
  // 32-byte (256-bit) accesses are legal for full chunks of: bit 0 out_f32, bit 1 out_f16,
  // bit 2 res_f32 (pointer 32-byte aligned, row pitch a multiple of 32 bytes); each one
  // sector per L2 request instead of half of one
  int32_t wide;
  uint32_t* err;
  // optional int8 residual added before the activation (same layout as the outputs):
  // y = (f32)acc * scale + (f32)r * res_scale
  const int8_t* residual;
  float res_scale;
  // convolution (ACB > 0)
  int32_t ow, ohw;           // output width, OH*OW
  int32_t sw, sh, pw, ph;    // stride / padding
  int32_t dw, dh, kw;        // dilation, filter width
  int32_t chunks_per_tap;    // C / ACB
  int32_t total_chunks;      // KH*KW*C / ACB
  // shared-memory plan (set by launch_cfg): a_stages A (or A+W) ring slots; w_resident = 1
  // keeps the whole [BN x K] weight tile in shared memory, loaded once per CTA (one N tile)
  int32_t a_stages;
  int32_t w_resident;
  // bounded-wait limit of the single-CTA kernel, and its test hook: when withhold_kb >= 0,
  // CTA 0 never issues the copies of k-block withhold_kb of its first tile (the waits on that
  // stage then run out after wait_ns and the launch reports LSC_ERROR_TIMEOUT)
  unsigned long long wait_ns = kWaitLimitNs;
  int32_t withhold_kb = -1;
  // 3x3 / 2 max pool (padding 1) fused into a pixel-grouped convolution (the CNN stem; the
  // POOL kernel variant): the grouped output is walked in bands of 4 conv rows
  // (band_rows = 4 * ow grouped pixels per tile, tiles of one image contiguous), each CTA a
  // contiguous range of bands; the band's int8 conv rows go to a five-row ring in shared
  // memory and the two pool rows they complete go to out_i8 ([N, ph_out, pw_out, cout]).
  int32_t band_rows, bands, pool_tiles;  // per tile, per image, in all
  int32_t conv_w, conv_h, cout, group;   // conv output width / height (ungrouped), channels, G
  int32_t ph_out, pw_out;
};

// The pool variant's ring of conv rows: 5 rows x conv_w pixels x cout int8 channels.  Its
// geometry is the ResNet stem's, fixed at compile time so that the epilogue's index arithmetic
// divides by constants (divisions by run-time values doubled the epilogue's instruction count):
// groups of 4 pixels, 64 channels, 112 conv columns (28 grouped), bands of 4 rows.
constexpr int kPoolRingRows = 5;
constexpr int kPoolG = 4, kPoolCout = 64, kPoolConvW = 112;
constexpr int kPoolOWG = kPoolConvW / kPoolG, kPoolBandRows = 4 * kPoolOWG, kPoolCQ = kPoolCout / 16;
constexpr int kPoolPW = kPoolConvW / 2;

constexpr int kSmemLimit = 232448;  // opt-in dynamic shared memory per block (227 KB)

// ---- several producer threads ------------------------------------------------------------
// One thread completes only about one TMA tensor load per ~600 cycles on B200, whatever the
// box size up to 64 KB (measured with lsc_probe_tma_rate: ~25 B/clk per SM with 16 KB boxes
// from one thread, ~97 B/clk from four), while a 128 x 256 x 32 int8 MMA takes 128 cycles.  So
// the loads of every k-block are spread over kProducers threads (lane 0 of each producer warp):
// load j of k-block iteration `it` (counted over the CTA's tiles in consumption order) belongs
// to producer (it * L + j) % kProducers, L = loads per k-block, and the producer of load 0
// posts the stage's byte count.  Another producer's bytes may land first; the mbarrier's
// tx-count then goes negative for a while, and the phase still completes only after that
// arrive.  A producer waits only on the slots it loads into, and the ring needs at least
// kProducers stages: a producer's loads are then less than a ring round apart, so its parity
// wait on `empty` cannot alias a phase two rounds back.  (Waiting on every slot does not lift
// that limit: a producer behind the others can then meet a slot two phases ahead and wait for
// a phase that needs its own load; measured on B200 as a bounded-wait timeout.)  The producers
// are lanes 0-1 of warps 0-1: separate threads are what matters (measured: two lanes of one
// warp deliver 44 B/clk, two warps 49), and 19 warps keep the 96 registers per thread that a
// fifth warp on one SM sub-partition (21 warps) would cut to 80.  Measured and not kept on
// B200: eight producers as lanes 0-3 of the same two warps (ResNet-18 step 1.087 -> 1.120 ms
// at batch 256, 0.275 -> 0.336 ms at batch 32: four lanes of one warp spinning on different
// barriers and issuing copies serialise each other), dealing the A loads round-robin over
// all four producers instead of two (4096^3 GEMM 2554 -> 2468 TOPS), and the producer count
// as a runtime value (its modulo in every iteration cost 3 % at batch 256, 12 % at batch 32:
// the producers set the pace of small-batch convolutions, which is also why the im2col tap
// coordinates come from a stepped cursor, TapCursor, instead of two divisions per load:
// 1.096 -> 1.083 ms at batch 256, 0.278 -> 0.268 ms at batch 32), and six producers as lanes
// 0-1 of three warps (20 warps, still 96 registers; loads dealt without divisions: 1.082 ->
// 1.094 ms at batch 256, 0.268 -> 0.276 ms at batch 32 -- the extra spinning warp takes issue
// slots from the MMA and epilogue warps of its sub-partition).
constexpr int kProducerWarps = 2;
constexpr int kProducerLanes = 2;
constexpr int kProducers = kProducerWarps * kProducerLanes;

// Shared-memory record the MMA warp reads to drain the loads still in flight after an abort.
struct ProducerLog {
  int32_t slot_it[8];  // the iteration whose loads were posted into each ring slot
  uint32_t done;       // producer threads that have left their loop
};

__device__ __forceinline__ void producer_log_init(ProducerLog* lg) {
  for (int i = 0; i < 8; ++i) lg->slot_it[i] = -1;
  lg->done = 0u;
}

// The owner of a k-block iteration's load 0, once every load of the iteration it took part in
// is issued, notes the iteration in the log; every producer leaving its loop counts itself out.
__device__ __forceinline__ void producer_leave(ProducerLog* lg) {
  __threadfence_block();
  atomicAdd(&lg->done, 1u);
}

// After an abort (MMA thread): waits (bounded) until every producer has left its loop, then for
// each of the `stages` iterations from it_next on whose loads were posted waits for them to
// land, so no copy is still writing shared memory when the CTA exits.
__device__ __noinline__ void drain_in_flight(uint64_t* full, int stages, int it_next, ProducerLog* lg,
                                             uint32_t* err, unsigned long long wait_ns) {
  volatile uint32_t* done = &lg->done;
  const unsigned long long t0 = globaltimer_ns();
  while (*done < static_cast<uint32_t>(kProducers)) {
    if (globaltimer_ns() - t0 > wait_ns) {
      if (err) atomicOr(err, LSC_DEVERR_TIMEOUT);
      break;
    }
  }
  volatile uint32_t no_abort = 0;
  volatile int32_t* slot_it = lg->slot_it;
  for (int d = 0; d < stages; ++d) {
    const int i = it_next + d;
    const int st = i % stages;
    if (slot_it[st] == i) mbar_wait(&full[st], static_cast<uint32_t>((i / stages) & 1), &no_abort, err, wait_ns);
  }
}

// Index, among this producer's loads of iteration `it`, of its first load (>= L: none).
__device__ __forceinline__ int first_load_of(int pr, int it, int L) {
  return (pr - (it * L) % kProducers + kProducers) % kProducers;
}

// Channel chunk jc of a convolution's K dimension, in (kh, kw, c) order, as (chunk within its
// tap, kx, ky), advanced one chunk at a time.  The producers keep one per tile and step it by
// the k-block's chunk count every iteration instead of dividing jc by the chunks per tap and
// the tap by KW: the producer threads set the pace of small-batch convolutions, and two
// integer divisions per load are a visible share of their time.
struct TapCursor {
  int ci = 0, kx = 0, ky = 0, jc = 0;
  __device__ __forceinline__ void step(int chunks_per_tap, int kw) {
    ++jc;
    if (++ci == chunks_per_tap) {
      ci = 0;
      if (++kx == kw) {
        kx = 0;
        ++ky;
      }
    }
  }
};

// The cursor `n` chunks past `c` (n < 8), or chunk 0 once past the filter (its weights are
// zero there, so any in-bounds load serves).
__device__ __forceinline__ TapCursor tap_at(TapCursor c, int n, const I8Params& p) {
  for (int t = 0; t < n; ++t) c.step(p.chunks_per_tap, p.kw);
  if (c.jc >= p.total_chunks) c = TapCursor{};
  return c;
}

template <int BN_>
struct I8Cfg {
  static constexpr int BM = 128;
  static constexpr int BN = BN_;
  static constexpr int BK = 128;  // int8 elements (= bytes) of K per stage
  static constexpr int STAGES = BN_ == 256 ? 4 : (BN_ == 128 ? 6 : 8);
  static constexpr int A_BYTES = BM * BK;
  static constexpr int B_BYTES = BN * BK;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TMEM_COLS = 2 * BN;  // two accumulator buffers; power of 2 >= 32
  // EPI_WARPS epilogue warps: EPI_WARPS / 4 per TMEM lane quarter, each taking that share of
  // the tile's columns in chunks of EPI_W
  static constexpr int EPI_WARPS = 16;
  static constexpr int MMA_WARP = kProducerWarps;  // producer warps, then the MMA warp, then epilogue
  static constexpr int THREADS = 32 * (kProducerWarps + 1 + EPI_WARPS);
  static constexpr int COLS_PER_EPI_WARP = BN / (EPI_WARPS / 4);
  static constexpr int EPI_W = 16;
  static constexpr int MAX_STAGES = 8;  // barrier slots
  static constexpr int RES_STAGES = 4;  // A ring depth when the weights are resident
  static constexpr int BAR_BYTES = 256;
  // per epilogue warp: the scale and bias of the columns it handles in the current N tile
  static constexpr int EPI_COL_BYTES = EPI_WARPS * COLS_PER_EPI_WARP * 8;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + BAR_BYTES + EPI_COL_BYTES;
  static constexpr uint32_t IDESC = idesc_i8(BM, BN);
  static_assert(SMEM_BYTES <= kSmemLimit, "shared memory budget");
  static_assert((2 * MAX_STAGES + 7) * 8 + 8 <= 192 && 192 + sizeof(ProducerLog) <= BAR_BYTES, "barrier area");
  static_assert(STAGES <= MAX_STAGES && STAGES >= kProducers && RES_STAGES >= kProducers, "ring slots");
  // shared memory with the weights resident: RES_STAGES A slots, kblocks W tiles
  static constexpr int res_smem_bytes(int kblocks) {
    return RES_STAGES * A_BYTES + kblocks * B_BYTES + 1024 + BAR_BYTES + EPI_COL_BYTES;
  }
};

// CTA-pair GEMM: 6 stages x (16 KB A + 16 KB W) per CTA; EPI_WARPS epilogue warps over the
// 256 accumulator columns in EPI_W-column chunks
struct PairCfg {
  static constexpr int STAGES = 6;
  static constexpr int EPI_WARPS = 16;
  static constexpr int EPI_W = 16;
  static constexpr int MMA_WARP = kProducerWarps;  // producer warps, the MMA warp, the epilogue
  static constexpr int THREADS = 32 * (kProducerWarps + 1 + EPI_WARPS);
  static constexpr int COLS_PER_EPI_WARP = 256 / (EPI_WARPS / 4);
  static constexpr int BAR_BYTES = 256;
  static constexpr int EPI_COL_BYTES = EPI_WARPS * COLS_PER_EPI_WARP * 8;
  static constexpr int SMEM_BYTES = STAGES * (2 * 128 * 128) + 1024 + BAR_BYTES + EPI_COL_BYTES;
  static_assert(SMEM_BYTES <= kSmemLimit, "shared memory budget");
  static constexpr int LOG_OFFSET = 160;  // ProducerLog within the barrier area
  static_assert((2 * STAGES + 5) * 8 + 8 <= LOG_OFFSET && LOG_OFFSET + sizeof(ProducerLog) <= BAR_BYTES,
                "barrier area");
  static_assert(STAGES >= kProducers, "ring slots");
};


// Pulls this thread's f32 residual segment for the coming tile into L2 (issued before the
// accumulator is ready, so the loads in the epilogue hit L2): `cols` columns from col0.
__device__ __forceinline__ void prefetch_residual(const I8Params& p, int row, int col0, int cols) {
  if (row >= p.m || !p.res_f32) return;
  const float* rp = p.res_f32 + static_cast<int64_t>(row) * p.ldo;
  for (int i = 0; i < cols; i += 32)
    if (col0 + i < p.n) asm volatile("prefetch.global.L2 [%0];" ::"l"(rp + col0 + i));
}

// This thread's 16 int8 residual values of columns [col0, col0 + 16) when the epilogue will read
// them as one vector (zero otherwise): loaded a chunk ahead, so the load's latency overlaps the
// accumulator's wait and the previous chunk's arithmetic instead of stalling the chunk.
__device__ __forceinline__ uint4 load_residual16(const I8Params& p, int row, int col0) {
  if (!p.residual || row >= p.m || !p.vec_ok || col0 + 16 > p.n) return make_uint4(0u, 0u, 0u, 0u);
  return __ldg(reinterpret_cast<const uint4*>(p.residual + static_cast<int64_t>(row) * p.ldo + col0));
}

// Epilogue for W consecutive columns of one output row held by this thread; cs / cb are the
// chunk's per-column scales and biases staged in shared memory (zero past the last column).
// Each output is stored as soon as it is final (i32, then f32, then int8) so the
// accumulator, f32 and int8 arrays are never live together.  EXT compiles in the f16 output
// and the f32 residual (the transformer projections); without them the CNN's kernels keep
// their registers and instructions for the int8 path.
template <int ACT, int W, bool EXT>
__device__ __forceinline__ void epilogue_chunk(const I8Params& p, const uint32_t (&r)[W],
                                               const float* cs, const int32_t* cb, int row, int col0,
                                               const uint4* res_pre = nullptr) {
  static_assert(W % 16 == 0, "chunks are whole 16-byte int8 vectors");
  if (row >= p.m) return;
  const bool vec = (col0 + W <= p.n) && p.vec_ok;
  const int64_t base = static_cast<int64_t>(row) * p.ldo + col0;
  int32_t acc[W];
#pragma unroll
  for (int j = 0; j < W; j += 4) {
    const int4 b = *reinterpret_cast<const int4*>(cb + j);
    acc[j + 0] = static_cast<int32_t>(r[j + 0] + static_cast<uint32_t>(b.x));
    acc[j + 1] = static_cast<int32_t>(r[j + 1] + static_cast<uint32_t>(b.y));
    acc[j + 2] = static_cast<int32_t>(r[j + 2] + static_cast<uint32_t>(b.z));
    acc[j + 3] = static_cast<int32_t>(r[j + 3] + static_cast<uint32_t>(b.w));
  }
  if (p.out_i32) {
    if (vec) {
      int4* dst = reinterpret_cast<int4*>(p.out_i32 + base);
#pragma unroll
      for (int j = 0; j < W / 4; ++j) dst[j] = make_int4(acc[4 * j], acc[4 * j + 1], acc[4 * j + 2], acc[4 * j + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < W; ++j)
        if (col0 + j < p.n) p.out_i32[base + j] = acc[j];
    }
  }
  if (!p.out_f32 && !p.out_i8 && !(EXT && p.out_f16)) return;
  float y[W];
#pragma unroll
  for (int j = 0; j < W; j += 4) {
    const float4 s = *reinterpret_cast<const float4*>(cs + j);
    f2unpack(f2mul(f2pack(__int2float_rn(acc[j]), __int2float_rn(acc[j + 1])), f2pack(s.x, s.y)), y[j], y[j + 1]);
    f2unpack(f2mul(f2pack(__int2float_rn(acc[j + 2]), __int2float_rn(acc[j + 3])), f2pack(s.z, s.w)), y[j + 2],
             y[j + 3]);
  }
  if (p.residual) {
    if (vec) {
#pragma unroll
      for (int v = 0; v < W / 16; ++v) {
        const uint4 rv = res_pre ? res_pre[v] : __ldg(reinterpret_cast<const uint4*>(p.residual + base) + v);
        const uint32_t rw[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int32_t q = static_cast<int8_t>((rw[j >> 2] >> (8 * (j & 3))) & 0xFFu);
          y[16 * v + j] = __fadd_rn(y[16 * v + j], __fmul_rn(__int2float_rn(q), p.res_scale));
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < W; ++j)
        if (col0 + j < p.n)
          y[j] = __fadd_rn(y[j], __fmul_rn(__int2float_rn(p.residual[base + j]), p.res_scale));
    }
  }
  if (EXT && p.res_f32) {
    if (vec && (p.wide & 4)) {
#pragma unroll
      for (int v = 0; v < W / 8; ++v) {
        uint32_t rv[8];
        ld_global_nc_v8(p.res_f32 + base + 8 * v, rv);
#pragma unroll
        for (int j = 0; j < 8; ++j) y[8 * v + j] = __fadd_rn(y[8 * v + j], __uint_as_float(rv[j]));
      }
    } else if (vec) {
      const float4* rp = reinterpret_cast<const float4*>(p.res_f32 + base);
#pragma unroll
      for (int v = 0; v < W / 4; ++v) {
        const float4 r4 = __ldg(rp + v);
        y[4 * v + 0] = __fadd_rn(y[4 * v + 0], r4.x);
        y[4 * v + 1] = __fadd_rn(y[4 * v + 1], r4.y);
        y[4 * v + 2] = __fadd_rn(y[4 * v + 2], r4.z);
        y[4 * v + 3] = __fadd_rn(y[4 * v + 3], r4.w);
      }
    } else {
#pragma unroll
      for (int j = 0; j < W; ++j)
        if (col0 + j < p.n) y[j] = __fadd_rn(y[j], p.res_f32[base + j]);
    }
  }
  // A ReLU feeding only the int8 output is applied inside the requantization's clamp.
  const bool relu_folded = ACT == LSC_ACT_RELU && !p.out_f32 && !(EXT && p.out_f16) && p.inv_s_out > 0.0f;
  if constexpr (ACT == LSC_ACT_GELU) {
#pragma unroll
    for (int j = 0; j < W; j += 2) act_gelu2(y[j], y[j + 1]);
  } else if (!relu_folded) {
#pragma unroll
    for (int j = 0; j < W; ++j) y[j] = apply_act<ACT>(y[j]);
  }
  if (p.out_f32) {
    if (vec && (p.wide & 1)) {
#pragma unroll
      for (int v = 0; v < W / 8; ++v) {
        uint32_t ov[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) ov[j] = __float_as_uint(y[8 * v + j]);
        st_global_v8(p.out_f32 + base + 8 * v, ov);
      }
    } else if (vec) {
      float4* dst = reinterpret_cast<float4*>(p.out_f32 + base);
#pragma unroll
      for (int j = 0; j < W / 4; ++j) dst[j] = make_float4(y[4 * j], y[4 * j + 1], y[4 * j + 2], y[4 * j + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < W; ++j)
        if (col0 + j < p.n) p.out_f32[base + j] = y[j];
    }
  }
  if (EXT && p.out_f16) {
    __half* o = p.out_f16 + base;
    if (vec && (p.wide & 2)) {
#pragma unroll
      for (int v = 0; v < W / 16; ++v) {
        uint32_t h[8];
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          const __half2 hh = __floats2half2_rn(y[16 * v + 2 * t], y[16 * v + 2 * t + 1]);
          h[t] = *reinterpret_cast<const uint32_t*>(&hh);
        }
        st_global_v8(o + 16 * v, h);
      }
    } else if (vec) {
#pragma unroll
      for (int v = 0; v < W / 8; ++v) {
        uint32_t h[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const __half2 hh = __floats2half2_rn(y[8 * v + 2 * t], y[8 * v + 2 * t + 1]);
          h[t] = *reinterpret_cast<const uint32_t*>(&hh);
        }
        reinterpret_cast<uint4*>(o)[v] = make_uint4(h[0], h[1], h[2], h[3]);
      }
    } else {
#pragma unroll
      for (int j = 0; j < W; ++j)
        if (col0 + j < p.n) o[j] = __float2half_rn(y[j]);
    }
  }
  if (p.out_i8) {
    uint32_t pk[W / 4];
    requant_pack<W>(y, p.s_out, p.inv_s_out, relu_folded, p.rounding, pk);
    if (vec) {
      uint4* dst = reinterpret_cast<uint4*>(p.out_i8 + base);
#pragma unroll
      for (int v = 0; v < W / 16; ++v) dst[v] = make_uint4(pk[4 * v], pk[4 * v + 1], pk[4 * v + 2], pk[4 * v + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < W; ++j)
        if (col0 + j < p.n) p.out_i8[base + j] = static_cast<int8_t>((pk[j >> 2] >> (8 * (j & 3))) & 0xFFu);
    }
  }
}

// Shared-memory descriptor of the A operand for the kk-th K=32 slice of a stage.
// ACB = 0: dense 128-byte rows (128-byte swizzle).  ACB > 0: the stage holds 128/ACB
// im2col sub-tiles of [128 rows x ACB bytes] with the swizzle that matches ACB.
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

// Ring address of 16 channels (group cq) of conv pixel (y, x): the 16-byte granules of a ring
// row are XOR-swizzled by the grouped column, so the 32 lanes of an epilogue warp (32
// consecutive grouped pixels, one pixel of each group) store to different banks.
__device__ __forceinline__ uint4* pool_ring_at(uint8_t* ring, int y, int x, int cq) {
  const int gx = x / kPoolG;
  const int gi = (x * kPoolCQ + cq) ^ (gx & 7);
  return reinterpret_cast<uint4*>(ring + (y % kPoolRingRows) * (kPoolConvW * kPoolCout)) + gi;
}

// The pool variant's epilogue for 16 accumulator columns of one grouped output row: the INT8
// chain's int8-only arithmetic (bias, scale, folded ReLU or the activation, requantize) with
// the codes written to the ring instead of global memory.
template <int ACT>
__device__ __forceinline__ void pool_chunk(const I8Params& p, const uint32_t (&r)[16], const float* cs,
                                           const int32_t* cb, int row_in_tile, int tcol, int band, uint8_t* ring) {
  if (row_in_tile >= kPoolBandRows) return;
  float y[16];
#pragma unroll
  for (int j = 0; j < 16; j += 4) {
    const int4 b = *reinterpret_cast<const int4*>(cb + j);
    const float4 sc = *reinterpret_cast<const float4*>(cs + j);
    const int32_t a0 = static_cast<int32_t>(r[j + 0] + static_cast<uint32_t>(b.x));
    const int32_t a1 = static_cast<int32_t>(r[j + 1] + static_cast<uint32_t>(b.y));
    const int32_t a2 = static_cast<int32_t>(r[j + 2] + static_cast<uint32_t>(b.z));
    const int32_t a3 = static_cast<int32_t>(r[j + 3] + static_cast<uint32_t>(b.w));
    f2unpack(f2mul(f2pack(__int2float_rn(a0), __int2float_rn(a1)), f2pack(sc.x, sc.y)), y[j], y[j + 1]);
    f2unpack(f2mul(f2pack(__int2float_rn(a2), __int2float_rn(a3)), f2pack(sc.z, sc.w)), y[j + 2], y[j + 3]);
  }
  const bool relu_folded = ACT == LSC_ACT_RELU && p.inv_s_out > 0.0f;
  if (!relu_folded) {
#pragma unroll
    for (int j = 0; j < 16; ++j) y[j] = apply_act<ACT>(y[j]);
  }
  uint32_t pk[4];
  requant_pack<16>(y, p.s_out, p.inv_s_out, relu_folded, p.rounding, pk);
  const int cr = row_in_tile / kPoolOWG, gx = row_in_tile - cr * kPoolOWG;
  const int g = tcol / kPoolCout, ch = tcol - g * kPoolCout;
  *pool_ring_at(ring, 4 * band + cr, gx * kPoolG + g, ch >> 4) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
}

// 3x3 / 2 max pool (padding 1, padding taps skipped) of the two pool rows band `band` of image
// n completes, from the ring to out_i8: work item i = (pool row of the two, pool column,
// 16-channel group); int8 codes compare like the values (one positive per-tensor scale).
__device__ __forceinline__ void pool_rows(const I8Params& p, uint8_t* ring, int n, int band, int tid, int nthreads) {
  constexpr int items = 2 * kPoolPW * kPoolCQ;
  for (int i = tid; i < items; i += nthreads) {
    const int prl = i / (kPoolPW * kPoolCQ);
    const int rem = i - prl * (kPoolPW * kPoolCQ);
    const int px = rem / kPoolCQ, cq = rem - px * kPoolCQ;
    const int py = 2 * band + prl;
    if (py >= p.ph_out) continue;
    uint4 m = make_uint4(0x80808080u, 0x80808080u, 0x80808080u, 0x80808080u);
#pragma unroll
    for (int dy = -1; dy <= 1; ++dy) {
      const int yy = 2 * py + dy;
      if (yy < 0 || yy >= p.conv_h) continue;
#pragma unroll
      for (int dx = -1; dx <= 1; ++dx) {
        const int xx = 2 * px + dx;
        if (xx < 0 || xx >= kPoolConvW) continue;
        const uint4 v = *pool_ring_at(ring, yy, xx, cq);
        m.x = __vmaxs4(m.x, v.x);
        m.y = __vmaxs4(m.y, v.y);
        m.z = __vmaxs4(m.z, v.z);
        m.w = __vmaxs4(m.w, v.w);
      }
    }
    reinterpret_cast<uint4*>(p.out_i8 + ((static_cast<int64_t>(n) * p.ph_out + py) * kPoolPW + px) * kPoolCout)[cq] = m;
  }
}

// The tiles a CTA walks: strided over the grid, or (pool variant) a contiguous range of bands,
// preceded by the band before it when that belongs to the same image -- its last conv row is
// the first pool row's upper window row.  `prefix` = that extra band's index (-1: none).
template <bool POOL>
__device__ __forceinline__ void cta_tiles(const I8Params& p, int num_tiles, int& begin, int& end, int& step,
                                          int& prefix) {
  if constexpr (POOL) {
    const int64_t T = p.pool_tiles, G = gridDim.x, b = blockIdx.x;
    begin = static_cast<int>((b * T) / G);
    end = static_cast<int>(((b + 1) * T) / G);
    prefix = -1;
    if (begin < end && begin % p.bands != 0) prefix = --begin;
    step = 1;
  } else {
    begin = blockIdx.x;
    end = num_tiles;
    step = gridDim.x;
    prefix = -1;
  }
}

template <int BN, int ACT, int ACB, bool EXT, bool POOL = false>
__global__ void __launch_bounds__(I8Cfg<BN>::THREADS, 1)
    contraction_i8_kernel(const __grid_constant__ CUtensorMap tmA,
                          const __grid_constant__ CUtensorMap tmW, const I8Params p) {
  using C = I8Cfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int kblocks = (p.k + C::BK - 1) / C::BK;
  const int stages = p.a_stages;
  const bool wres = p.w_resident != 0;
  // [A ring: stages x A_BYTES][W: stages (ring) or kblocks (resident) x B_BYTES][barriers][epi]
  uint8_t* sA = smem;
  uint8_t* sW = smem + stages * C::A_BYTES;
  uint8_t* after_w = sW + (wres ? kblocks : stages) * C::B_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(after_w);
  uint64_t* full = bars;
  uint64_t* empty = bars + C::MAX_STAGES;
  uint64_t* tfull = bars + 2 * C::MAX_STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* wfull = drain + 1;  // resident weights landed
  uint64_t* pbar = wfull + 1;   // pool variant: the epilogue warps' band barrier
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(pbar + 1);
  volatile uint32_t* abort_flag = tmem_slot + 1;
  ProducerLog* plog = reinterpret_cast<ProducerLog*>(after_w + 192);
  uint8_t* epi_cols = after_w + C::BAR_BYTES;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::MAX_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], C::EPI_WARPS);
    }
    mbar_init(drain, 1);
    mbar_init(wfull, kProducers);
    mbar_init(pbar, C::EPI_WARPS);
    *abort_flag = 0u;
    producer_log_init(plog);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmW);
  }
  if (warp == C::MMA_WARP) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // the next kernel on the stream may now be scheduled onto SMs this grid leaves
  griddep_launch_dependents();

  const int m_tiles = (p.m + C::BM - 1) / C::BM;
  const int n_tiles = (p.n + C::BN - 1) / C::BN;
  const int num_tiles = m_tiles * n_tiles;
  int t_begin, t_end, t_step, t_prefix;
  cta_tiles<POOL>(p, num_tiles, t_begin, t_end, t_step, t_prefix);

  if (warp < kProducerWarps) {
    if (lane < kProducerLanes) {
      // ------------------------------------------------------------- TMA producers
      const int pr = warp * kProducerLanes + lane;
      bool ok = true;
      if (wres) {
        // the whole weight tile (one N tile: nb = 0) once, on its own barrier, spread over the
        // producers; the weights are constant, so they are requested before the wait for the
        // previous kernel
        uint32_t mine = 0;
        for (int kb = pr; kb < kblocks; kb += kProducers) mine += C::B_BYTES;
        mbar_arrive_expect_tx(wfull, mine);
        for (int kb = pr; kb < kblocks; kb += kProducers) tma_load_2d(&tmW, wfull, sW + kb * C::B_BYTES, kb * C::BK, 0);
      }
      griddep_wait();  // A is the previous kernel's output
      constexpr int SUB = ACB > 0 ? 128 / ACB : 1;  // A loads per k-block
      const int L = SUB + (wres ? 0 : 1);          // then the W load
      const uint32_t stage_bytes = wres ? C::A_BYTES : C::STAGE_BYTES;
      int it = 0;
      int ring_stage = 0;  // it % stages and (it / stages) & 1, kept incrementally
      uint32_t ring_phase = 0;
      for (int tile = t_begin; tile < t_end && ok; tile += t_step) {
        const int mb = POOL ? 0 : tile % m_tiles, nb = POOL ? 0 : tile / m_tiles;
        // filter-origin coordinates of the tile's first output pixel (convolution only)
        int32_t cw = 0, chh = 0, cn = 0;
        if constexpr (ACB > 0) {
          const int m0 = POOL ? tile * p.band_rows : mb * C::BM;
          cn = m0 / p.ohw;
          const int rem = m0 - cn * p.ohw;
          const int oy = rem / p.ow;
          const int ox = rem - oy * p.ow;
          cw = ox * p.sw - p.pw;
          chh = oy * p.sh - p.ph;
        }
        TapCursor cur;  // chunk kb * SUB (convolution only)
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int stage = ring_stage;
          const uint32_t phase = ring_phase;
          if (++ring_stage == stages) {
            ring_stage = 0;
            ring_phase ^= 1u;
          }
          const TapCursor base = cur;
          if constexpr (ACB > 0) {
#pragma unroll
            for (int t = 0; t < SUB; ++t) cur.step(p.chunks_per_tap, p.kw);
          }
          const int j0 = first_load_of(pr, it, L);
          if (j0 >= L) continue;
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, p.err, p.wait_ns)) {
            ok = false;
            break;
          }
          // test hook: the loads of this k-block are never issued, so nothing completes `full`
          if (p.withhold_kb == kb && blockIdx.x == 0 && tile == static_cast<int>(blockIdx.x)) continue;
          if (j0 == 0) mbar_arrive_expect_tx(&full[stage], stage_bytes);
          uint8_t* a_dst = sA + stage * C::A_BYTES;
          for (int j = j0; j < L; j += kProducers) {
            if (j == SUB) {
              tma_load_2d(&tmW, &full[stage], sW + stage * C::B_BYTES, kb * C::BK, nb * C::BN);
            } else if constexpr (ACB == 0) {
              tma_load_2d(&tmA, &full[stage], a_dst, kb * C::BK, mb * C::BM);
            } else {
              const TapCursor c = tap_at(base, j, p);  // chunk kb * SUB + j
              tma_load_im2col_4d(&tmA, &full[stage], a_dst + j * (C::BM * ACB), c.ci * ACB, cw, chh, cn,
                                 static_cast<uint16_t>(c.kx * p.dw), static_cast<uint16_t>(c.ky * p.dh));
            }
          }
          if (j0 == 0) plog->slot_it[stage] = it;
        }
      }
      producer_leave(plog);
    }
  } else if (warp == C::MMA_WARP) {
    // --------------------------------------------------------------- MMA issuer
    // The whole warp runs the loop, waits together and agrees on the outcome (__all_sync); one
    // elected lane issues.  Measured on B200: a lone lane issuing tcgen05.mma while the rest of
    // its warp is parked takes ~450 cycles per k-block of four, the converged warp ~370.
    // Shared-memory descriptors are the stage-0 descriptors plus the byte offset / 16 in their
    // start-address field (shared addresses stay below 2^18, so the field cannot carry).
    int it = 0;
    int stage = 0;  // it % stages and (it / stages) & 1, kept incrementally
    uint32_t phase = 0;
    int local = 0;
    bool ok = true;
    bool any_mma = false;
    uint64_t a_kk[C::BK / 32], w_kk[C::BK / 32];
#pragma unroll
    for (int kk = 0; kk < C::BK / 32; ++kk) {
      a_kk[kk] = a_desc<ACB>(smem_u32(sA), kk);
      w_kk[kk] = smem_desc_sw128_kmajor(smem_u32(sW) + kk * 32);
    }
    if (wres) ok = __all_sync(0xFFFFFFFFu, mbar_wait(wfull, 0u, abort_flag, p.err, p.wait_ns));
    for (int tile = t_begin; tile < t_end && ok; tile += t_step, ++local) {
      const int buf = local & 1;
      const uint32_t buf_phase = static_cast<uint32_t>((local >> 1) & 1);
      ok = __all_sync(0xFFFFFFFFu, mbar_wait(&tempty[buf], buf_phase ^ 1u, abort_flag, p.err, p.wait_ns));
      if (!ok) break;
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * C::BN);
      for (int kb = 0; kb < kblocks; ++kb, ++it) {
        ok = __all_sync(0xFFFFFFFFu, mbar_wait(&full[stage], phase, abort_flag, p.err, p.wait_ns));
        if (!ok) break;
        tc_fence_after();
        const uint64_t ao = static_cast<uint64_t>(stage * (C::A_BYTES >> 4));
        const uint64_t wo = static_cast<uint64_t>((wres ? kb : stage) * (C::B_BYTES >> 4));
        if (elect_one()) {
#pragma unroll
          for (int kk = 0; kk < C::BK / 32; ++kk)
            mma_i8(d_tmem, a_kk[kk] + ao, w_kk[kk] + wo, C::IDESC, (kb | kk) != 0 ? 1u : 0u);
          mma_commit(&empty[stage]);
        }
        __syncwarp();
        any_mma = true;
        if (++stage == stages) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (ok) {
        if (elect_one()) mma_commit(&tfull[buf]);
        __syncwarp();
      }
    }
    if (!ok) {
      // Let the copies in flight land and the MMAs already issued finish before TMEM and the
      // shared memory are released.
      if (elect_one()) {
        drain_in_flight(full, stages, it, plog, p.err, p.wait_ns);
        volatile uint32_t no_abort = 0;
        if (wres) mbar_wait(wfull, 0u, &no_abort, p.err, p.wait_ns);
        if (any_mma) {
          mma_commit(drain);
          mbar_wait(drain, 0u, &no_abort, p.err, p.wait_ns);
        }
      }
      __syncwarp();
    }
  } else {
    // --------------------------------------------------------------- epilogue
    const int epi = warp - C::MMA_WARP - 1;  // 0..EPI_WARPS-1
    const int quarter = warp & 3;   // TMEM lane quarter this warp may read
    const int part = epi >> 2;      // which share of the tile's columns
    const int row_in_tile = quarter * 32 + lane;
    // this warp's column scales / biases: [COLS_PER_EPI_WARP] floats then as many int32
    float* w_scale = reinterpret_cast<float*>(epi_cols + epi * (C::COLS_PER_EPI_WARP * 8));
    int32_t* w_bias = reinterpret_cast<int32_t*>(w_scale + C::COLS_PER_EPI_WARP);
    int staged_nb = -1;
    int local = 0;
    uint8_t* ring = epi_cols + C::EPI_COL_BYTES;  // the pool variant's conv rows
    uint32_t pool_ph = 0;
    // the pool variant's band barrier over the epilogue warps: an mbarrier with a bounded wait,
    // so a warp that gave up on a wait cannot leave the others blocked
    auto band_sync = [&]() -> bool {
      __syncwarp();
      if (lane == 0) mbar_arrive(pbar);
      const bool ok = mbar_wait(pbar, pool_ph, abort_flag, p.err, p.wait_ns);
      pool_ph ^= 1u;
      return ok;
    };
    griddep_wait();  // outputs and the residual belong to earlier kernels until they finish
    for (int tile = t_begin; tile < t_end; tile += t_step, ++local) {
      const int mb = POOL ? 0 : tile % m_tiles, nb = POOL ? 0 : tile / m_tiles;
      if (nb != staged_nb) {
        __syncwarp();
        for (int i = lane; i < C::COLS_PER_EPI_WARP; i += 32) {
          const int col = nb * C::BN + part * C::COLS_PER_EPI_WARP + i;
          w_scale[i] = col < p.n ? __ldg(p.scale + col) : 0.0f;
          w_bias[i] = (p.bias && col < p.n) ? __ldg(p.bias + col) : 0;
        }
        __syncwarp();
        staged_nb = nb;
      }
      const int buf = local & 1;
      const uint32_t buf_phase = static_cast<uint32_t>((local >> 1) & 1);
      const int row = POOL ? tile * p.band_rows + row_in_tile : mb * C::BM + row_in_tile;
      if constexpr (EXT) prefetch_residual(p, row, nb * C::BN + part * C::COLS_PER_EPI_WARP, C::COLS_PER_EPI_WARP);
      static_assert(C::EPI_W == 16, "one 16-byte residual vector per chunk");
      const int col_first = nb * C::BN + part * C::COLS_PER_EPI_WARP;
      uint4 res_next = load_residual16(p, row, col_first);  // before the accumulator is ready
      if (!mbar_wait(&tfull[buf], buf_phase, abort_flag, p.err, p.wait_ns)) break;
      tc_fence_after();
      constexpr int CHUNKS = C::COLS_PER_EPI_WARP / C::EPI_W;
#pragma unroll 1
      for (int c = 0; c < CHUNKS; ++c) {
        const int tcol = part * C::COLS_PER_EPI_WARP + c * C::EPI_W;
        const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                               static_cast<uint32_t>(buf * C::BN + tcol);
        uint32_t r[C::EPI_W];
        tmem_ld_cols(taddr, r);
        const uint4 res_cur = res_next;
        if (c + 1 < CHUNKS) res_next = load_residual16(p, row, col_first + (c + 1) * C::EPI_W);
        tmem_ld_wait();
        if (c == CHUNKS - 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tempty[buf]);
        }
        if constexpr (POOL) {
          pool_chunk<ACT>(p, r, w_scale + c * C::EPI_W, w_bias + c * C::EPI_W, row_in_tile, tcol, tile % p.bands, ring);
        } else {
          epilogue_chunk<ACT, C::EPI_W, EXT>(p, r, w_scale + c * C::EPI_W, w_bias + c * C::EPI_W, row,
                                             nb * C::BN + tcol, &res_cur);
        }
      }
      if constexpr (POOL) {
        // every epilogue warp's rows of the band are in the ring: pool the two rows they
        // complete (not for the prefix band, whose pool rows belong to the CTA before), then
        // keep the ring until all reads are done
        if (!band_sync()) break;
        if (tile != t_prefix) pool_rows(p, ring, tile / p.bands, tile % p.bands, epi * 32 + lane, 32 * C::EPI_WARPS);
        if (!band_sync()) break;
      }
    }
  }

  __syncthreads();
  if (warp == C::MMA_WARP) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// ------------------------------------------------------------------------------------------
// CTA-pair GEMM (cluster of 2, tcgen05 cta_group::2) for large dense contractions.
//
// A pair owns a 256 x 256 output tile.  Each CTA fetches its own 128 rows of A and its own
// 128 of the tile's 256 W rows (no multicast), so a pair moves 512 rows of operands per
// 65,536 outputs where two independent 128 x 256 CTAs move 768.  The even CTA issues
// tcgen05.mma.cta_group::2 (M = 256, N = 256, K = 32) over both CTAs' shared memory; each
// CTA's TMEM receives its 128 rows x 256 columns, double-buffered (512 columns).
//   producer (warp 0, both CTAs): waits on its own `empty` slot, loads A and W halves with
//     completion counted on the even CTA's `full` barrier (the even producer posts the
//     pair's byte count);
//   MMA (warp 1, even CTA): waits `full`, issues 4 MMAs per stage, commits the stage to
//     both CTAs' `empty` and the finished tile to both CTAs' `tfull` (multicast commit);
//   epilogue (warps 2-17, both CTAs): as the single-CTA kernel on the CTA's own rows; the
//     last TMEM read of a tile arrives on the even CTA's `tempty` (2 x 16 arrivals).
// All waits are bounded; both CTAs meet at a cluster barrier before TMEM is released.
template <int PN, int ACT, bool EXT>
__global__ void __launch_bounds__(PairCfg::THREADS, 1)
    contraction_i8_pair_kernel(const __grid_constant__ CUtensorMap tmA,
                               const __grid_constant__ CUtensorMap tmW, const I8Params p) {
  using C = I8Cfg<256>;  // BK
  using P = PairCfg;
  constexpr int ROWS = 128;                   // A rows per CTA
  constexpr int WROWS = PN / 2;               // W rows per CTA (the pair tile is 256 x PN)
  constexpr int STAGES = PairCfg::STAGES;
  constexpr int A_BYTES = ROWS * C::BK;
  constexpr int W_BYTES = 128 * C::BK;        // stage slot (WROWS rows used)
  constexpr uint32_t IDESC = idesc_i8(256, PN);
  constexpr int COLS = PN / (P::EPI_WARPS / 4);  // accumulator columns per epilogue warp
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sW = smem + STAGES * A_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sW + STAGES * W_BYTES);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* tfull = bars + 2 * STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile uint32_t* abort_flag = tmem_slot + 1;
  ProducerLog* plog = reinterpret_cast<ProducerLog*>(reinterpret_cast<uint8_t*>(bars) + P::LOG_OFFSET);
  uint8_t* epi_cols = reinterpret_cast<uint8_t*>(bars) + P::BAR_BYTES;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool even = rank == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 2 * P::EPI_WARPS);
    }
    mbar_init(drain, 1);
    *abort_flag = 0u;
    producer_log_init(plog);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmW);
  }
  if (warp == P::MMA_WARP) {
    tmem_alloc_pair(tmem_slot, 2 * PN);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers initialised before any remote arrive / complete_tx
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t full_even = mapa_shared(smem_u32(full), 0);
  const uint32_t tempty_even = mapa_shared(smem_u32(tempty), 0);
  griddep_launch_dependents();

  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int m_tiles = (p.m + 255) / 256;
  const int n_tiles = (p.n + PN - 1) / PN;
  const int num_tiles = m_tiles * n_tiles;
  const int kblocks = (p.k + C::BK - 1) / C::BK;

  if (warp < kProducerWarps) {
    if (lane < kProducerLanes) {
      // ------------------------------------------------------------- TMA producers (both CTAs)
      // Each CTA loads its own halves; they complete on the even CTA's `full`, where the even
      // CTA's owner of load 0 posts the pair's byte count.
      const int pr = warp * kProducerLanes + lane;
      bool ok = true;
      griddep_wait();  // A is the previous kernel's output
      constexpr int L = 2;  // A rows, W rows
      int it = 0;
      int ring_stage = 0;
      uint32_t ring_phase = 0;
      for (int tile = pair; tile < num_tiles && ok; tile += npairs) {
        const int mb = tile % m_tiles, nb = tile / m_tiles;
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int stage = ring_stage;
          const uint32_t phase = ring_phase;
          if (++ring_stage == STAGES) {
            ring_stage = 0;
            ring_phase ^= 1u;
          }
          const int j0 = first_load_of(pr, it, L);
          if (j0 >= L) continue;
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, p.err)) {
            ok = false;
            break;
          }
          if (even && j0 == 0) mbar_arrive_expect_tx(&full[stage], 2 * (A_BYTES + WROWS * C::BK));
          const uint32_t fb = full_even + stage * 8;
          for (int j = j0; j < L; j += kProducers) {
            if (j == 0)
              tma_load_2d_pair(&tmA, fb, sA + stage * A_BYTES, kb * C::BK, mb * 256 + static_cast<int>(rank) * ROWS);
            else
              tma_load_2d_pair(&tmW, fb, sW + stage * W_BYTES, kb * C::BK, nb * PN + static_cast<int>(rank) * WROWS);
          }
          if (j0 == 0) plog->slot_it[stage] = it;
        }
      }
      producer_leave(plog);
    }
  } else if (warp == P::MMA_WARP) {
    if (even) {
      // ----------------------------------------------------------- MMA issuer (even CTA, converged warp)
      int it = 0;
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      bool any_mma = false;
      uint64_t a_kk[C::BK / 32], w_kk[C::BK / 32];
#pragma unroll
      for (int kk = 0; kk < C::BK / 32; ++kk) {
        a_kk[kk] = smem_desc_sw128_kmajor(smem_u32(sA) + kk * 32);
        w_kk[kk] = smem_desc_sw128_kmajor(smem_u32(sW) + kk * 32);
      }
      for (int tile = pair; tile < num_tiles && ok; tile += npairs, ++local) {
        const int buf = local & 1;
        const uint32_t buf_phase = static_cast<uint32_t>((local >> 1) & 1);
        ok = __all_sync(0xFFFFFFFFu, mbar_wait(&tempty[buf], buf_phase ^ 1u, abort_flag, p.err));
        if (!ok) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * PN);
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          ok = __all_sync(0xFFFFFFFFu, mbar_wait(&full[stage], phase, abort_flag, p.err));
          if (!ok) break;
          tc_fence_after();
          const uint64_t ao = static_cast<uint64_t>(stage * (A_BYTES >> 4));
          const uint64_t wo = static_cast<uint64_t>(stage * (W_BYTES >> 4));
          if (elect_one()) {
#pragma unroll
            for (int kk = 0; kk < C::BK / 32; ++kk)
              mma_i8_pair(d_tmem, a_kk[kk] + ao, w_kk[kk] + wo, IDESC, (kb | kk) != 0 ? 1u : 0u);
            mma_commit_pair(&empty[stage], 0x3);
          }
          __syncwarp();
          any_mma = true;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (ok) {
          if (elect_one()) mma_commit_pair(&tfull[buf], 0x3);
          __syncwarp();
        }
      }
      if (!ok) {
        // the pair's copies in flight complete on these barriers; the MMAs issued must finish
        if (elect_one()) {
          drain_in_flight(full, STAGES, it, plog, p.err, kWaitLimitNs);
          if (any_mma) {
            volatile uint32_t no_abort = 0;
            mma_commit_pair(drain, 0x1);
            mbar_wait(drain, 0u, &no_abort, p.err);
          }
        }
        __syncwarp();
      }
    }
  } else {
    // --------------------------------------------------------------- epilogue (own rows)
    const int epi = warp - P::MMA_WARP - 1;
    const int quarter = warp & 3;
    const int part = epi >> 2;
    const int row_in_tile = quarter * 32 + lane;
    float* w_scale = reinterpret_cast<float*>(epi_cols + epi * (COLS * 8));
    int32_t* w_bias = reinterpret_cast<int32_t*>(w_scale + COLS);
    int staged_nb = -1;
    int local = 0;
    griddep_wait();  // outputs and the residual belong to earlier kernels until they finish
    for (int tile = pair; tile < num_tiles; tile += npairs, ++local) {
      const int mb = tile % m_tiles, nb = tile / m_tiles;
      if (nb != staged_nb) {
        __syncwarp();
        for (int i = lane; i < COLS; i += 32) {
          const int col = nb * PN + part * COLS + i;
          w_scale[i] = col < p.n ? __ldg(p.scale + col) : 0.0f;
          w_bias[i] = (p.bias && col < p.n) ? __ldg(p.bias + col) : 0;
        }
        __syncwarp();
        staged_nb = nb;
      }
      const int buf = local & 1;
      const uint32_t buf_phase = static_cast<uint32_t>((local >> 1) & 1);
      const int row = mb * 256 + static_cast<int>(rank) * ROWS + row_in_tile;
      if constexpr (EXT) prefetch_residual(p, row, nb * PN + part * COLS, COLS);
      if (!mbar_wait(&tfull[buf], buf_phase, abort_flag, p.err)) break;
      tc_fence_after();
      constexpr int CHUNKS = COLS / P::EPI_W;
#pragma unroll 1
      for (int c = 0; c < CHUNKS; ++c) {
        const int tcol = part * COLS + c * P::EPI_W;
        const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                               static_cast<uint32_t>(buf * PN + tcol);
        uint32_t r[P::EPI_W];
        tmem_ld_cols(taddr, r);
        tmem_ld_wait();
        if (c == CHUNKS - 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(tempty_even + buf * 8);
        }
        epilogue_chunk<ACT, P::EPI_W, EXT>(p, r, w_scale + c * P::EPI_W, w_bias + c * P::EPI_W, row,
                                           nb * PN + tcol);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no CTA leaves while its peer may still signal its barriers
  if (warp == P::MMA_WARP) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, 2 * PN);
  }
}

template <int BN, int ACT, int ACB, bool EXT>
lsc_status launch_cfg(const CUtensorMap& ta, const CUtensorMap& tw, const I8Params& p,
                      const DeviceState& ds, cudaStream_t stream) {
  using C = I8Cfg<BN>;
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [] {
    attr_err = cudaFuncSetAttribute(contraction_i8_kernel<BN, ACT, ACB, EXT>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
  });
  if (attr_err != cudaSuccess) return cuda_error(attr_err, "cudaFuncSetAttribute(contraction_i8)");
  const int m_tiles = (p.m + C::BM - 1) / C::BM;
  const int n_tiles = (p.n + C::BN - 1) / C::BN;
  const int tiles = m_tiles * n_tiles;
  const int grid = tiles < ds.sm_count ? tiles : ds.sm_count;
  // Keep the weights resident when there is a single N tile, they fit beside a RES_STAGES A
  // ring, and each CTA runs several M tiles (so the one-time load is amortised): the W tile
  // then crosses L2 once per CTA instead of once per M tile.
  const int kblocks = (p.k + C::BK - 1) / C::BK;
  I8Params q = p;
  q.w_resident = (n_tiles == 1 && m_tiles >= 2 * grid && C::res_smem_bytes(kblocks) <= kSmemLimit) ? 1 : 0;
  q.a_stages = q.w_resident ? C::RES_STAGES : C::STAGES;
  const int smem = q.w_resident ? C::res_smem_bytes(kblocks) : C::SMEM_BYTES;
  LSC_CUDA_TRY(launch_dependent(ds.overlap_launches, contraction_i8_kernel<BN, ACT, ACB, EXT>, dim3(grid), dim3(C::THREADS),
                                smem, stream, ta, tw, q));
  return LSC_SUCCESS;
}

// The pool variant (the CNN stem: BN = 256 grouped columns, 64-byte channel blocks, ReLU):
// weights resident, the deepest A ring that fits beside them and the ring of conv rows.
lsc_status launch_pool_cfg(const CUtensorMap& ta, const CUtensorMap& tw, const I8Params& p, const DeviceState& ds,
                           cudaStream_t stream) {
  using C = I8Cfg<256>;
  auto kernel = contraction_i8_kernel<256, LSC_ACT_RELU, 64, false, true>;
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [kernel] {
    attr_err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
  });
  if (attr_err != cudaSuccess) return cuda_error(attr_err, "cudaFuncSetAttribute(contraction_i8 pool)");
  const int kblocks = (p.k + C::BK - 1) / C::BK;
  const int ring = kPoolRingRows * p.conv_w * p.cout;
  int stages = C::RES_STAGES;
  auto smem_of = [&](int st) { return st * C::A_BYTES + kblocks * C::B_BYTES + 1024 + C::BAR_BYTES + C::EPI_COL_BYTES + ring; };
  while (stages > 2 && smem_of(stages) > kSmemLimit) --stages;
  if (smem_of(stages) > kSmemLimit)
    return set_error(LSC_ERROR_UNSUPPORTED_OPERATOR, "conv_pool_i8: filter and row ring exceed shared memory");
  I8Params q = p;
  q.w_resident = 1;
  q.a_stages = stages;
  const int grid = p.pool_tiles < ds.sm_count ? p.pool_tiles : ds.sm_count;
  LSC_CUDA_TRY(launch_dependent(ds.overlap_launches, kernel, dim3(grid), dim3(C::THREADS), smem_of(stages), stream,
                                ta, tw, q));
  return LSC_SUCCESS;
}

template <int BN, int ACB, bool EXT>
lsc_status launch_act(const CUtensorMap& ta, const CUtensorMap& tw, const I8Params& p, int act,
                      const DeviceState& ds, cudaStream_t stream) {
  switch (act) {
    case LSC_ACT_RELU: return launch_cfg<BN, LSC_ACT_RELU, ACB, EXT>(ta, tw, p, ds, stream);
    case LSC_ACT_RELU6: return launch_cfg<BN, LSC_ACT_RELU6, ACB, EXT>(ta, tw, p, ds, stream);
    case LSC_ACT_SILU: return launch_cfg<BN, LSC_ACT_SILU, ACB, EXT>(ta, tw, p, ds, stream);
    case LSC_ACT_GELU: return launch_cfg<BN, LSC_ACT_GELU, ACB, EXT>(ta, tw, p, ds, stream);
    default: return launch_cfg<BN, LSC_ACT_NONE, ACB, EXT>(ta, tw, p, ds, stream);
  }
}

// Launch of the CTA-pair kernel: clusters of 2, one pair per two SMs up to the number of
// pairs the device can hold at once (persistent over 256 x 256 tiles).
template <int PN, int ACT, bool EXT>
lsc_status launch_pair_act(const CUtensorMap& ta, const CUtensorMap& tw, const I8Params& p, const DeviceState& ds,
                           cudaStream_t stream) {
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  static int max_pairs = 0;
  std::call_once(once, [&ds] {
    attr_err = cudaFuncSetAttribute(contraction_i8_pair_kernel<PN, ACT, EXT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    PairCfg::SMEM_BYTES);
    if (attr_err != cudaSuccess) return;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(static_cast<unsigned>(ds.sm_count & ~1));
    cfg.blockDim = dim3(PairCfg::THREADS);
    cfg.dynamicSmemBytes = PairCfg::SMEM_BYTES;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    attr_err = cudaOccupancyMaxActiveClusters(&max_pairs, contraction_i8_pair_kernel<PN, ACT, EXT>, &cfg);
  });
  if (attr_err != cudaSuccess) return cuda_error(attr_err, "contraction_i8_pair setup");
  if (max_pairs < 1) return set_error(LSC_ERROR_EXECUTION_FAILED, "gemm_i8: no CTA pair fits on the device");
  const int tiles = ((p.m + 255) / 256) * ((p.n + PN - 1) / PN);
  const int pairs = tiles < max_pairs ? tiles : max_pairs;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // see launch_dependent
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs));
  cfg.blockDim = dim3(PairCfg::THREADS);
  cfg.dynamicSmemBytes = PairCfg::SMEM_BYTES;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = ds.overlap_launches ? 2 : 1;
  LSC_CUDA_TRY(cudaLaunchKernelEx(&cfg, contraction_i8_pair_kernel<PN, ACT, EXT>, ta, tw, p));
  return LSC_SUCCESS;
}

template <bool EXT>
lsc_status launch_pair(const CUtensorMap& ta, const CUtensorMap& tw, const I8Params& p, int act, const DeviceState& ds,
                       cudaStream_t stream) {
  switch (act) {
    case LSC_ACT_RELU: return launch_pair_act<256, LSC_ACT_RELU, EXT>(ta, tw, p, ds, stream);
    case LSC_ACT_RELU6: return launch_pair_act<256, LSC_ACT_RELU6, EXT>(ta, tw, p, ds, stream);
    case LSC_ACT_SILU: return launch_pair_act<256, LSC_ACT_SILU, EXT>(ta, tw, p, ds, stream);
    case LSC_ACT_GELU: return launch_pair_act<256, LSC_ACT_GELU, EXT>(ta, tw, p, ds, stream);
    default: return launch_pair_act<256, LSC_ACT_NONE, EXT>(ta, tw, p, ds, stream);
  }
}

template <int ACB, bool EXT = false>
lsc_status launch_bn(int bn, const CUtensorMap& ta, const CUtensorMap& tw, const I8Params& p,
                     int act, const DeviceState& ds, cudaStream_t stream) {
  switch (bn) {
    case 64: return launch_act<64, ACB, EXT>(ta, tw, p, act, ds, stream);
    case 128: return launch_act<128, ACB, EXT>(ta, tw, p, act, ds, stream);
    default: return launch_act<256, ACB, EXT>(ta, tw, p, act, ds, stream);
  }
}

// ------------------------------------------------------------------------------------------
// Convolution with the operands swapped, for layers of exactly 128 output channels: the
// filter is the 128-row A operand (TMEM lanes = output channels) and 256 output pixels, two
// 128-pixel im2col loads per channel block, are the N = 256 B operand (TMEM columns =
// pixels).  A K = 32 int8 MMA costs about the same at N = 128 as at N = 256 on B200, so
// putting the pixels on the wide side does up to twice the work per instruction of the
// 128 x 128 tiles the plain kernel uses for these layers.  The epilogue works per output
// channel (one per thread); the four warps sharing a pixel range pass each 16-pixel x
// 128-channel int8 block through a 2 KB shared-memory stage so that global accesses are
// 16-byte pixel-row segments.  Same arithmetic, same bits.
struct SwapCfg {
  static constexpr int BM = 128;   // output channels (A rows)
  static constexpr int BP = 256;   // output pixels per tile (B rows)
  static constexpr int BK = 128;
  static constexpr int STAGES = 4;
  static constexpr int W_BYTES = BM * BK;
  static constexpr int X_BYTES = BP * BK;
  static constexpr int STAGE_BYTES = W_BYTES + X_BYTES;
  static constexpr int EPI_WARPS = 16;
  static constexpr int MMA_WARP = kProducerWarps;  // producer warps, the MMA warp, the epilogue
  static constexpr int THREADS = 32 * (kProducerWarps + 1 + EPI_WARPS);
  static constexpr int TMEM_COLS = 2 * BP;  // double-buffered accumulator
  static constexpr int BAR_BYTES = 256;
  static constexpr int OUT_STAGE_BYTES = 4 * 2048;  // per part: 16 pixels x 128 channels of int8
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + BAR_BYTES + OUT_STAGE_BYTES;
  static constexpr uint32_t IDESC = idesc_i8(BM, BP);
  static_assert(SMEM_BYTES <= kSmemLimit, "shared memory budget");
  static constexpr int LOG_OFFSET = 128;  // ProducerLog within the barrier area
  static_assert((2 * STAGES + 5) * 8 + 8 <= LOG_OFFSET && LOG_OFFSET + sizeof(ProducerLog) <= BAR_BYTES,
                "barrier area");
  static_assert(STAGES >= kProducers, "ring slots");
};

template <int ACB>
__device__ __forceinline__ uint64_t swap_x_desc(uint32_t x0, int kk) {
  if constexpr (ACB == 128) {
    return smem_desc_sw128_kmajor(x0 + kk * 32);
  } else {
    static_assert(ACB == 64, "swapped convolutions take 64- or 128-byte channel blocks");
    return smem_desc_sw64_kmajor(x0 + (kk >> 1) * (SwapCfg::BP * 64) + (kk & 1) * 32);
  }
}

template <int ACT, int ACB, int RND>
__global__ void __launch_bounds__(SwapCfg::THREADS, 1)
    contraction_i8_swap_kernel(const __grid_constant__ CUtensorMap tmX,
                               const __grid_constant__ CUtensorMap tmW, const I8Params p) {
  using S = SwapCfg;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sW = smem;                             // [stages][128 rows][128 B]
  uint8_t* sX = smem + S::STAGES * S::W_BYTES;    // [stages][chunks][256 rows][ACB]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::STAGES * S::STAGE_BYTES);
  uint64_t* full = bars;
  uint64_t* empty = bars + S::STAGES;
  uint64_t* tfull = bars + 2 * S::STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile uint32_t* abort_flag = tmem_slot + 1;
  ProducerLog* plog = reinterpret_cast<ProducerLog*>(reinterpret_cast<uint8_t*>(bars) + S::LOG_OFFSET);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int kblocks = (p.k + S::BK - 1) / S::BK;
  const int num_tiles = (p.m + S::BP - 1) / S::BP;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S::STAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], S::EPI_WARPS);
    }
    mbar_init(drain, 1);
    *abort_flag = 0u;
    producer_log_init(plog);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmX);
    tma_prefetch_desc(&tmW);
  }
  if (warp == S::MMA_WARP) {
    tmem_alloc(tmem_slot, S::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  griddep_launch_dependents();

  if (warp < kProducerWarps) {
    if (lane < kProducerLanes) {
      // ------------------------------------------------------------- TMA producers
      const int pr = warp * kProducerLanes + lane;
      bool ok = true;
      griddep_wait();  // the activations are the previous kernel's output
      constexpr int SUB = 128 / ACB;
      constexpr int L = 1 + 2 * SUB;  // the filter block, then two 128-pixel halves per channel block
      int it = 0;
      int ring_stage = 0;
      uint32_t ring_phase = 0;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        // filter-origin coordinates of each 128-pixel half's first pixel
        int32_t cw[2], chh[2], cn[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int m0 = tile * S::BP + h * 128;
          cn[h] = m0 / p.ohw;
          const int rem = m0 - cn[h] * p.ohw;
          const int oy = rem / p.ow;
          const int ox = rem - oy * p.ow;
          cw[h] = ox * p.sw - p.pw;
          chh[h] = oy * p.sh - p.ph;
        }
        TapCursor cur;  // chunk kb * SUB
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int stage = ring_stage;
          const uint32_t phase = ring_phase;
          if (++ring_stage == S::STAGES) {
            ring_stage = 0;
            ring_phase ^= 1u;
          }
          const TapCursor base = cur;
#pragma unroll
          for (int t = 0; t < SUB; ++t) cur.step(p.chunks_per_tap, p.kw);
          const int j0 = first_load_of(pr, it, L);
          if (j0 >= L) continue;
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, p.err)) {
            ok = false;
            break;
          }
          if (j0 == 0) mbar_arrive_expect_tx(&full[stage], S::STAGE_BYTES);
          uint8_t* x_dst = sX + stage * S::X_BYTES;
          for (int j = j0; j < L; j += kProducers) {
            if (j == 0) {
              tma_load_2d(&tmW, &full[stage], sW + stage * S::W_BYTES, kb * S::BK, 0);
            } else {
              const int i = (j - 1) >> 1, h = (j - 1) & 1;
              const TapCursor c = tap_at(base, i, p);  // chunk kb * SUB + i
              tma_load_im2col_4d(&tmX, &full[stage], x_dst + i * (S::BP * ACB) + h * (128 * ACB), c.ci * ACB, cw[h],
                                 chh[h], cn[h], static_cast<uint16_t>(c.kx * p.dw), static_cast<uint16_t>(c.ky * p.dh));
            }
          }
          if (j0 == 0) plog->slot_it[stage] = it;
        }
      }
      producer_leave(plog);
    }
  } else if (warp == S::MMA_WARP) {
    // ------------------------------------------------------------- MMA issuer (converged warp, one elected lane)
    int it = 0;
    int stage = 0;
    uint32_t phase = 0;
    int local = 0;
    bool ok = true, any_mma = false;
    uint64_t w_kk[S::BK / 32], x_kk[S::BK / 32];
#pragma unroll
    for (int kk = 0; kk < S::BK / 32; ++kk) {
      w_kk[kk] = smem_desc_sw128_kmajor(smem_u32(sW) + kk * 32);
      x_kk[kk] = swap_x_desc<ACB>(smem_u32(sX), kk);
    }
    for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++local) {
      const int buf = local & 1;
      ok = __all_sync(0xFFFFFFFFu, mbar_wait(&tempty[buf], static_cast<uint32_t>((local >> 1) & 1) ^ 1u, abort_flag,
                                             p.err));
      if (!ok) break;
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * S::BP);
      for (int kb = 0; kb < kblocks; ++kb, ++it) {
        ok = __all_sync(0xFFFFFFFFu, mbar_wait(&full[stage], phase, abort_flag, p.err));
        if (!ok) break;
        tc_fence_after();
        const uint64_t wo = static_cast<uint64_t>(stage * (S::W_BYTES >> 4));
        const uint64_t xo = static_cast<uint64_t>(stage * (S::X_BYTES >> 4));
        if (elect_one()) {
#pragma unroll
          for (int kk = 0; kk < S::BK / 32; ++kk)
            mma_i8(d_tmem, w_kk[kk] + wo, x_kk[kk] + xo, S::IDESC, (kb | kk) != 0 ? 1u : 0u);
          mma_commit(&empty[stage]);
        }
        __syncwarp();
        any_mma = true;
        if (++stage == S::STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (ok) {
        if (elect_one()) mma_commit(&tfull[buf]);
        __syncwarp();
      }
    }
    if (!ok) {
      if (elect_one()) {
        drain_in_flight(full, S::STAGES, it, plog, p.err, kWaitLimitNs);
        if (any_mma) {
          volatile uint32_t no_abort = 0;
          mma_commit(drain);
          mbar_wait(drain, 0u, &no_abort, p.err);
        }
      }
      __syncwarp();
    }
  } else {
    // --------------------------------------------------------------- epilogue (one channel)
    const int epi = warp - S::MMA_WARP - 1;
    const int quarter = warp & 3;  // TMEM lane quarter this warp may read
    const int part = epi >> 2;     // which 64 of the tile's 256 pixels
    const int ch = quarter * 32 + lane;
    const int t = (epi & 3) * 32 + lane;  // thread index within the part (0..127)
    uint8_t* stage = smem + S::STAGES * S::STAGE_BYTES + S::BAR_BYTES + part * 2048;
    const uint32_t bar_id = 1u + static_cast<uint32_t>(part);
    const float scale = __ldg(p.scale + ch);  // p.n == 128: every channel exists
    const int32_t bias = p.bias ? __ldg(p.bias + ch) : 0;
    griddep_wait();  // outputs and the residual belong to earlier kernels until they finish
    int local = 0;
    const int srow = t >> 3, scol = (t & 7) * 16;  // this thread's 16 bytes of a pixel row
    // this thread's residual bytes of chunk c of `tile`, loaded a chunk ahead so the load's
    // latency overlaps the chunk before (the first chunk's before the accumulator is ready)
    auto residual_at = [&](int tile_, int c_) -> uint4 {
      const int px = tile_ * S::BP + part * 64 + c_ * 16 + srow;
      if (!p.residual || px >= p.m) return make_uint4(0u, 0u, 0u, 0u);
      return __ldg(reinterpret_cast<const uint4*>(p.residual + static_cast<int64_t>(px) * p.ldo + scol));
    };
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      const int buf = local & 1;
      uint4 res_next = residual_at(tile, 0);
      if (!mbar_wait(&tfull[buf], static_cast<uint32_t>((local >> 1) & 1), abort_flag, p.err)) break;
      tc_fence_after();
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                             static_cast<uint32_t>(buf * S::BP + part * 64);
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        const int col = part * 64 + c * 16;
        const int pix0 = tile * S::BP + col;
        uint32_t r[16];
        tmem_ld_cols(t_row + static_cast<uint32_t>(c * 16), r);
        tmem_ld_wait();
        if (c == 3) {
          // every accumulator column of the tile has been read
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tempty[buf]);
        }
        const uint4 res_cur = res_next;
        if (c < 3) res_next = residual_at(tile, c + 1);
        const bool srow_ok = pix0 + srow < p.m;
        int32_t acc[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) acc[j] = static_cast<int32_t>(r[j] + static_cast<uint32_t>(bias));
        if (p.out_i32) {
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (pix0 + j < p.m) p.out_i32[static_cast<int64_t>(pix0 + j) * p.ldo + ch] = acc[j];
        }
        if (!p.out_f32 && !p.out_i8) continue;
        float y[16];
        const uint64_t sc2 = f2pack(scale, scale);
#pragma unroll
        for (int j = 0; j < 16; j += 2)
          f2unpack(f2mul(f2pack(__int2float_rn(acc[j]), __int2float_rn(acc[j + 1])), sc2), y[j], y[j + 1]);
        if (p.residual) {
          // pixel rows in, channel columns out: 16-byte loads, then each lane its 16 bytes
          *reinterpret_cast<uint4*>(stage + srow * 128 + scol) = res_cur;
          named_bar_sync(bar_id, 128);
#pragma unroll
          for (int j = 0; j < 16; ++j)
            y[j] = __fadd_rn(y[j], __fmul_rn(__int2float_rn(static_cast<int32_t>(static_cast<int8_t>(stage[j * 128 + ch]))),
                                             p.res_scale));
          named_bar_sync(bar_id, 128);
        }
        // a ReLU feeding only the int8 output is applied inside the requantization's clamp
        const bool relu_folded = ACT == LSC_ACT_RELU && !p.out_f32 && p.inv_s_out > 0.0f;
        if (!relu_folded) {
#pragma unroll
          for (int j = 0; j < 16; ++j) y[j] = apply_act<ACT>(y[j]);
        }
        if (p.out_f32) {
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (pix0 + j < p.m) p.out_f32[static_cast<int64_t>(pix0 + j) * p.ldo + ch] = y[j];
        }
        if (p.out_i8) {
          uint32_t pk[4];  // pk[q]: pixels 4q .. 4q+3 of this channel, one byte each
          requant_pack_rnd<16, RND>(y, p.s_out, p.inv_s_out, relu_folded, pk);
          uint32_t* st32 = reinterpret_cast<uint32_t*>(stage);  // [pixel quad][channel]
#pragma unroll
          for (int q = 0; q < 4; ++q) st32[q * 128 + ch] = pk[q];
          named_bar_sync(bar_id, 128);
          // byte (srow & 3) of the 16 words of channels scol .. scol+15 in quad srow / 4
          const uint32_t* row = st32 + (srow >> 2) * 128 + scol;
          const uint32_t sel = static_cast<uint32_t>(srow & 3);
          uint32_t o[4];
#pragma unroll
          for (int w = 0; w < 4; ++w) {
            const uint32_t b0 = row[4 * w + 0], b1 = row[4 * w + 1], b2 = row[4 * w + 2], b3 = row[4 * w + 3];
            const uint32_t lo = __byte_perm(b0, b1, sel | ((sel + 4) << 4));
            const uint32_t hi = __byte_perm(b2, b3, sel | ((sel + 4) << 4));
            o[w] = __byte_perm(lo, hi, 0x5410);
          }
          if (srow_ok)
            *reinterpret_cast<uint4*>(p.out_i8 + static_cast<int64_t>(pix0 + srow) * p.ldo + scol) =
                make_uint4(o[0], o[1], o[2], o[3]);
          named_bar_sync(bar_id, 128);
        }
      }
    }
  }

  __syncthreads();
  if (warp == S::MMA_WARP) {
    tc_fence_after();
    tmem_dealloc(tmem_base, S::TMEM_COLS);
  }
}

template <int ACT, int ACB, int RND>
lsc_status launch_swap_cfg(const CUtensorMap& tx, const CUtensorMap& tw, const I8Params& p, const DeviceState& ds,
                           cudaStream_t stream) {
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [] {
    attr_err = cudaFuncSetAttribute(contraction_i8_swap_kernel<ACT, ACB, RND>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, SwapCfg::SMEM_BYTES);
  });
  if (attr_err != cudaSuccess) return cuda_error(attr_err, "cudaFuncSetAttribute(contraction_i8_swap)");
  const int tiles = (p.m + SwapCfg::BP - 1) / SwapCfg::BP;
  const int grid = tiles < ds.sm_count ? tiles : ds.sm_count;
  LSC_CUDA_TRY(launch_dependent(ds.overlap_launches, contraction_i8_swap_kernel<ACT, ACB, RND>, dim3(grid),
                                dim3(SwapCfg::THREADS), SwapCfg::SMEM_BYTES, stream, tx, tw, p));
  return LSC_SUCCESS;
}

template <int ACB, int RND>
lsc_status launch_swap_act(const CUtensorMap& tx, const CUtensorMap& tw, const I8Params& p, int act,
                           const DeviceState& ds, cudaStream_t stream) {
  switch (act) {
    case LSC_ACT_RELU: return launch_swap_cfg<LSC_ACT_RELU, ACB, RND>(tx, tw, p, ds, stream);
    case LSC_ACT_RELU6: return launch_swap_cfg<LSC_ACT_RELU6, ACB, RND>(tx, tw, p, ds, stream);
    case LSC_ACT_SILU: return launch_swap_cfg<LSC_ACT_SILU, ACB, RND>(tx, tw, p, ds, stream);
    default: return launch_swap_cfg<LSC_ACT_NONE, ACB, RND>(tx, tw, p, ds, stream);
  }
}

template <int ACB>
lsc_status launch_swap(const CUtensorMap& tx, const CUtensorMap& tw, const I8Params& p, int act,
                       const DeviceState& ds, cudaStream_t stream) {
  if (p.rounding == LSC_ROUND_HALF_EVEN) return launch_swap_act<ACB, LSC_ROUND_HALF_EVEN>(tx, tw, p, act, ds, stream);
  return launch_swap_act<ACB, LSC_ROUND_HALF_AWAY>(tx, tw, p, act, ds, stream);
}

// Column tile width: the widest tile that does not waste most of its columns.
// Column-tile width: the widest of 256/128/64 that does not waste a partial tile, narrowed
// while the grid would leave most SMs idle (small M, e.g. a classifier layer).
int pick_bn(int64_t m, int64_t n, int sm_count) {
  int bn;
  if (n <= 64) bn = 64;
  else if (n <= 128) bn = 128;
  else if (n % 256 == 0 || n % 128 != 0) bn = 256;
  else bn = 128;
  const int64_t m_tiles = (m + 127) / 128;
  while (bn > 64 && m_tiles * ((n + bn - 1) / bn) * 2 <= sm_count) bn /= 2;
  return bn;
}

// CTA-pair tile width for a GEMM (256), or 0 for single CTAs.  Pairs need N > 256 (a single
// N tile runs best weight-resident on single CTAs) and at least 32 pair tiles; measured on
// B200, a 256 x 256 pair tile beats both single-CTA tiles and 256 x 128 pair tiles even when
// there are fewer tiles than pairs (4096 x 1024 x 4096: 20.9 us against 30.1 us).
int pair_tile_n(int64_t m, int64_t n) {
  if (n <= 256 || m < 256) return 0;
  const int64_t t256 = ((m + 255) / 256) * ((n + 255) / 256);
  return t256 >= 32 ? 256 : 0;
}

lsc_status check_common(int64_t m, int64_t n, int act, int rounding, const float* scale,
                        int8_t* out_i8, float* out_f32, int32_t* out_i32, const char* who,
                        const void* out_f16 = nullptr) {
  if (m < 0 || n < 0) return set_error(LSC_ERROR_INVALID_ARGUMENT, "%s: negative size", who);
  if (!out_i8 && !out_f32 && !out_i32 && !out_f16)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "%s: no output given", who);
  if (m > 0 && n > 0 && !scale) return set_error(LSC_ERROR_INVALID_ARGUMENT, "%s: null scale", who);
  if (act < LSC_ACT_NONE || act > LSC_ACT_GELU)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "%s: bad activation %d", who, act);
  if (rounding != LSC_ROUND_HALF_AWAY && rounding != LSC_ROUND_HALF_EVEN)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "%s: bad rounding %d", who, rounding);
  return LSC_SUCCESS;
}

void fill_outputs(I8Params& p, const int32_t* bias, const float* scale, float s_out, int rounding,
                  int8_t* out_i8, float* out_f32, int32_t* out_i32, int64_t ldo, uint32_t* err) {
  p.bias = bias;
  p.scale = scale;
  p.s_out = s_out;
  const float inv = 1.0f / s_out;
  p.inv_s_out = (std::isnormal(s_out) && std::isnormal(inv)) ? inv : 0.0f;
  p.rounding = rounding;
  p.out_i8 = out_i8;
  p.out_f32 = out_f32;
  p.out_i32 = out_i32;
  p.ldo = ldo;
  const uintptr_t align_bits = reinterpret_cast<uintptr_t>(out_i8) |
                               reinterpret_cast<uintptr_t>(out_f32) |
                               reinterpret_cast<uintptr_t>(out_i32) |
                               reinterpret_cast<uintptr_t>(scale) |
                               reinterpret_cast<uintptr_t>(bias);
  p.vec_ok = ((align_bits & 15) == 0 && (ldo % 16) == 0) ? 1 : 0;
  p.wide = (p.vec_ok && (reinterpret_cast<uintptr_t>(out_f32) & 31) == 0 && ldo % 8 == 0) ? 1 : 0;
  p.err = err;
}

// Test hook of the bounded waits (lsc_debug_withhold_copy): the next `launches` INT8 GEMM
// launches on this thread that run on the single-CTA kernel withhold one operand copy and
// wait at most wait_ns.
struct WithholdRequest {
  int32_t launches = 0;
  unsigned long long wait_ns = kWaitLimitNs;
};
thread_local WithholdRequest t_withhold;

}  // namespace

lsc_status launch_gemm_i8(const int8_t* a, const int8_t* w, int64_t m, int64_t n, int64_t k,
                          const int32_t* bias, const float* scale, float s_out, int act,
                          int rounding, int8_t* out_i8, float* out_f32, int32_t* out_i32,
                          int64_t ldo, cudaStream_t stream, const GemmExtras* extras) {
  lsc_status st = check_common(m, n, act, rounding, scale, out_i8, out_f32, out_i32, "gemm_i8",
                               extras ? extras->out_f16 : nullptr);
  if (st) return st;
  if (m > INT32_MAX / 2 || n > INT32_MAX / 2 || k > INT32_MAX / 2)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "gemm_i8: size too large");
  if (m == 0 || n == 0) return LSC_SUCCESS;
  if (!a || !w) return set_error(LSC_ERROR_INVALID_ARGUMENT, "gemm_i8: null operand");
  if (k <= 0 || k % 16 != 0)
    return set_error(LSC_ERROR_INVALID_ARGUMENT,
                     "gemm_i8: K must be a positive multiple of 16 (got %lld)", (long long)k);
  if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(w)) & 15)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "gemm_i8: A and W must be 16-byte aligned");
  if (ldo < n) return set_error(LSC_ERROR_INVALID_ARGUMENT, "gemm_i8: ldo < n");
  DeviceState* ds = current_device_state();
  if (!ds) return LSC_ERROR_DEVICE_ERROR;
  if (ds->cc_major != 10)
    return set_error(LSC_ERROR_BACKEND_NOT_AVAILABLE,
                     "gemm_i8: needs an sm_100 (B200) device, found sm_%d%d", ds->cc_major,
                     ds->cc_minor);

  // CTA pairs for GEMMs wide and tall enough to give every pair of SMs 256 x 256 tiles;
  // single CTAs (128 x BN tiles) otherwise.
  const int pn = pair_tile_n(m, n);
  const bool pair = pn > 0;
  const int bn = pair ? pn / 2 : pick_bn(m, n, ds->sm_count);  // W box rows (a pair CTA holds PN/2)
  CUtensorMap ta, tw;
  st = encode_tmap_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, a, k, m, k, 128, 128,
                      CU_TENSOR_MAP_SWIZZLE_128B);
  if (st) return st;
  st = encode_tmap_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, w, k, n, k, 128, bn,
                      CU_TENSOR_MAP_SWIZZLE_128B);
  if (st) return st;

  I8Params p{};
  p.m = static_cast<int32_t>(m);
  p.n = static_cast<int32_t>(n);
  p.k = static_cast<int32_t>(k);
  fill_outputs(p, bias, scale, s_out, rounding, out_i8, out_f32, out_i32, ldo, ds->err_word);
  if (extras) {
    p.out_f16 = static_cast<__half*>(extras->out_f16);
    p.res_f32 = extras->res_f32;
    if ((reinterpret_cast<uintptr_t>(p.out_f16) | reinterpret_cast<uintptr_t>(p.res_f32)) & 15) p.vec_ok = 0;
    if (!p.vec_ok) {
      p.wide = 0;
    } else {
      if (p.out_f16 && (reinterpret_cast<uintptr_t>(p.out_f16) & 31) == 0 && ldo % 16 == 0) p.wide |= 2;
      if (p.res_f32 && (reinterpret_cast<uintptr_t>(p.res_f32) & 31) == 0 && ldo % 8 == 0) p.wide |= 4;
    }
  }
  if (!pair && t_withhold.launches > 0) {
    --t_withhold.launches;
    p.withhold_kb = 0;
    p.wait_ns = t_withhold.wait_ns;
  }
  if (p.out_f16 || p.res_f32) {
    if (pair) return launch_pair<true>(ta, tw, p, act, *ds, stream);
    return launch_bn<0, true>(bn, ta, tw, p, act, *ds, stream);
  }
  if (pair) return launch_pair<false>(ta, tw, p, act, *ds, stream);
  return launch_bn<0>(bn, ta, tw, p, act, *ds, stream);
}

lsc_status launch_conv_i8(const int8_t* x, const int8_t* w, const ConvGeometry& g,
                          const int32_t* bias, const float* scale, float s_out, int act,
                          int rounding, int8_t* out_i8, float* out_f32, int32_t* out_i32,
                          const int8_t* residual, float res_scale, cudaStream_t stream) {
  const int64_t m = g.n * g.oh * g.ow;
  lsc_status st = check_common(m, g.c_out, act, rounding, scale, out_i8, out_f32, out_i32, "conv_i8");
  if (st) return st;
  if (g.n < 0 || g.h <= 0 || g.w <= 0 || g.c <= 0 || g.kh <= 0 || g.kw <= 0 || g.sh <= 0 ||
      g.sw <= 0 || g.dh <= 0 || g.dw <= 0 || g.ph < 0 || g.pw < 0 || g.ph_b < -g.h || g.pw_r < -g.w)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "conv_i8: bad geometry");
  const int64_t span_h = g.h + g.ph + g.ph_b - g.dh * (g.kh - 1) - 1;
  const int64_t span_w = g.w + g.pw + g.pw_r - g.dw * (g.kw - 1) - 1;
  if (span_h < 0 || span_w < 0 || g.oh != span_h / g.sh + 1 || g.ow != span_w / g.sw + 1)
    return set_error(LSC_ERROR_SHAPE_MISMATCH, "conv_i8: output size does not match the geometry");
  if (g.c % 16 != 0)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "conv_i8: stored channels must be a multiple of 16 (got %lld)",
                     (long long)g.c);
  if (g.sh > 8 || g.sw > 8 || g.ph > 128 || g.pw > 128 || g.ph_b > 127 || g.pw_r > 127 ||
      g.ph_b - (g.kh - 1) * g.dh < -128 || g.pw_r - (g.kw - 1) * g.dw < -128 ||
      (g.kh - 1) * g.dh > 65535 || (g.kw - 1) * g.dw > 65535)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "conv_i8: stride/padding/filter outside the im2col unit's range");
  if (m == 0 || g.c_out == 0) return LSC_SUCCESS;
  if (m > INT32_MAX / 2 || g.n * g.h * g.w * g.c > (int64_t(1) << 40))
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "conv_i8: problem too large");
  if (!x || !w) return set_error(LSC_ERROR_INVALID_ARGUMENT, "conv_i8: null operand");
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w)) & 15)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "conv_i8: x and w must be 16-byte aligned");
  DeviceState* ds = current_device_state();
  if (!ds) return LSC_ERROR_DEVICE_ERROR;
  if (ds->cc_major != 10)
    return set_error(LSC_ERROR_BACKEND_NOT_AVAILABLE, "conv_i8: needs an sm_100 (B200) device");

  const int acb = g.c % 128 == 0 ? 128 : (g.c % 64 == 0 ? 64 : (g.c % 32 == 0 ? 32 : 16));
  const int64_t k = g.kh * g.kw * g.c;
  const uint64_t dims[4] = {static_cast<uint64_t>(g.c), static_cast<uint64_t>(g.w),
                            static_cast<uint64_t>(g.h), static_cast<uint64_t>(g.n)};
  const uint64_t strides[3] = {static_cast<uint64_t>(g.c), static_cast<uint64_t>(g.w * g.c),
                               static_cast<uint64_t>(g.h * g.w * g.c)};
  const int lower[2] = {static_cast<int>(-g.pw), static_cast<int>(-g.ph)};
  const int upper[2] = {static_cast<int>(g.pw_r - (g.kw - 1) * g.dw),
                        static_cast<int>(g.ph_b - (g.kh - 1) * g.dh)};
  const uint32_t estr[4] = {1, static_cast<uint32_t>(g.sw), static_cast<uint32_t>(g.sh), 1};
  const CUtensorMapSwizzle swz = acb == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                 : acb == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                 : acb == 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                                             : CU_TENSOR_MAP_SWIZZLE_NONE;
  CUtensorMap ta, tw;
  st = encode_tmap_im2col(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, x, dims, strides, lower, upper,
                          static_cast<uint32_t>(acb), 128, estr, swz);
  if (st) return st;
  const int bn = pick_bn(m, g.c_out, ds->sm_count);
  st = encode_tmap_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, w, static_cast<uint64_t>(k),
                      static_cast<uint64_t>(g.c_out), static_cast<uint64_t>(k), 128, bn,
                      CU_TENSOR_MAP_SWIZZLE_128B);
  if (st) return st;

  I8Params p{};
  p.m = static_cast<int32_t>(m);
  p.n = static_cast<int32_t>(g.c_out);
  const int64_t total_chunks = g.kh * g.kw * (g.c / acb);
  const int64_t sub = 128 / acb;
  p.k = static_cast<int32_t>(((total_chunks + sub - 1) / sub) * 128);
  p.ow = static_cast<int32_t>(g.ow);
  p.ohw = static_cast<int32_t>(g.oh * g.ow);
  p.sw = static_cast<int32_t>(g.sw);
  p.sh = static_cast<int32_t>(g.sh);
  p.pw = static_cast<int32_t>(g.pw);
  p.ph = static_cast<int32_t>(g.ph);
  p.dw = static_cast<int32_t>(g.dw);
  p.dh = static_cast<int32_t>(g.dh);
  p.kw = static_cast<int32_t>(g.kw);
  p.chunks_per_tap = static_cast<int32_t>(g.c / acb);
  p.total_chunks = static_cast<int32_t>(total_chunks);
  fill_outputs(p, bias, scale, s_out, rounding, out_i8, out_f32, out_i32, g.c_out, ds->err_word);
  p.residual = residual;
  p.res_scale = res_scale;
  if (reinterpret_cast<uintptr_t>(residual) & 15) p.vec_ok = 0;
  if (!p.vec_ok) p.wide = 0;
  // exactly 128 output channels, at least two k-blocks and two waves of 256-pixel tiles: the
  // operand-swapped kernel (pixels on the wide side of every MMA; the filter map's 128-row
  // box serves as its A operand).  Measured on B200 at batch 256: layer1 convs 98 -> 85 us,
  // layer2 3x3 convs 52-56 -> 43-52 us; a single k-block (the 1x1 downsample) or fewer than
  // two waves (layer1 at batch 32) run faster on the plain kernel.
  // The swap kernel's epilogue has no f16 output and no f32 residual: a convolution that asks
  // for either stays on the plain kernel.
  if (g.c_out == 128 && bn == 128 && p.vec_ok && (acb == 128 || acb == 64) && act != LSC_ACT_GELU &&
      !p.out_f16 && !p.res_f32 && p.k >= 256 && (m + 255) / 256 >= 2 * ds->sm_count) {
    if (acb == 128) return launch_swap<128>(ta, tw, p, act, *ds, stream);
    return launch_swap<64>(ta, tw, p, act, *ds, stream);
  }
  switch (acb) {
    case 128: return launch_bn<128>(bn, ta, tw, p, act, *ds, stream);
    case 64: return launch_bn<64>(bn, ta, tw, p, act, *ds, stream);
    case 32: return launch_bn<32>(bn, ta, tw, p, act, *ds, stream);
    default: return launch_bn<16>(bn, ta, tw, p, act, *ds, stream);
  }
}

lsc_status launch_conv_pool_i8(const int8_t* x, const int8_t* w, const ConvGeometry& g, int group,
                               const int32_t* bias, const float* scale, float s_out, int act, int rounding,
                               int8_t* out_pool, cudaStream_t stream) {
  const int64_t m = g.n * g.oh * g.ow;
  lsc_status st = check_common(m, g.c_out, act, rounding, scale, out_pool, nullptr, nullptr, "conv_pool_i8");
  if (st) return st;
  const int64_t cout = group > 0 ? g.c_out / group : 0;
  const int64_t conv_w = g.ow * group, conv_h = g.oh;
  if (act != LSC_ACT_RELU || g.c_out != 256 || group != kPoolG || cout != kPoolCout || conv_w != kPoolConvW ||
      g.c % 128 == 0 || g.c % 64 != 0 || g.sh != 1 || g.sw != 1 || g.dh != 1 || g.dw != 1 || conv_h % 4 ||
      !(s_out > 0.0f))
    return set_error(LSC_ERROR_UNSUPPORTED_OPERATOR,
                     "conv_pool_i8: the CNN stem's geometry only (4-pixel groups of 64 channels, 112 output columns, "
                     "64-byte channel blocks, stride 1, output height a multiple of 4, ReLU, int8 output)");
  const int64_t span_h = g.h + g.ph + g.ph_b - (g.kh - 1) - 1;
  const int64_t span_w = g.w + g.pw + g.pw_r - (g.kw - 1) - 1;
  if (g.n <= 0 || span_h < 0 || span_w < 0 || g.oh != span_h + 1 || g.ow != span_w + 1 || g.ph > 128 || g.pw > 128 ||
      g.ph_b > 127 || g.pw_r > 127 || g.ph_b - (g.kh - 1) < -128 || g.pw_r - (g.kw - 1) < -128)
    return set_error(LSC_ERROR_SHAPE_MISMATCH, "conv_pool_i8: output size does not match the geometry");
  if (m > INT32_MAX / 2 || g.n * g.h * g.w * g.c > (int64_t(1) << 40))
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "conv_pool_i8: problem too large");
  if (!x || !w || ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w) |
                    reinterpret_cast<uintptr_t>(out_pool)) & 15))
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "conv_pool_i8: x, w and the output must be 16-byte aligned");
  DeviceState* ds = current_device_state();
  if (!ds) return LSC_ERROR_DEVICE_ERROR;
  if (ds->cc_major != 10) return set_error(LSC_ERROR_BACKEND_NOT_AVAILABLE, "conv_pool_i8: needs an sm_100 (B200) device");
  // Bands of 4 rows fill 112 of a tile's 128 rows, and a CTA whose range starts inside an
  // image recomputes the band before it: with fewer than 16 bands per CTA that costs more than
  // the separate max pool (measured on B200: batch 256 1.0765 -> 1.0712 ms fused, batch 32
  // 0.2667 -> 0.2730 ms)
  if (g.n * (conv_h / 4) < 16 * static_cast<int64_t>(ds->sm_count))
    return set_error(LSC_ERROR_UNSUPPORTED_OPERATOR, "conv_pool_i8: too few bands per CTA to gain from the fusion");
  constexpr int acb = 64;
  const int64_t k = g.kh * g.kw * g.c;
  const uint64_t dims[4] = {static_cast<uint64_t>(g.c), static_cast<uint64_t>(g.w),
                            static_cast<uint64_t>(g.h), static_cast<uint64_t>(g.n)};
  const uint64_t strides[3] = {static_cast<uint64_t>(g.c), static_cast<uint64_t>(g.w * g.c),
                               static_cast<uint64_t>(g.h * g.w * g.c)};
  const int lower[2] = {static_cast<int>(-g.pw), static_cast<int>(-g.ph)};
  const int upper[2] = {static_cast<int>(g.pw_r - (g.kw - 1)), static_cast<int>(g.ph_b - (g.kh - 1))};
  const uint32_t estr[4] = {1, 1, 1, 1};
  CUtensorMap ta, tw;
  st = encode_tmap_im2col(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, x, dims, strides, lower, upper, acb, 128, estr,
                          CU_TENSOR_MAP_SWIZZLE_64B);
  if (st) return st;
  st = encode_tmap_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, w, static_cast<uint64_t>(k), 256, static_cast<uint64_t>(k),
                      128, 256, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st) return st;
  I8Params p{};
  p.m = static_cast<int32_t>(m);
  p.n = 256;
  const int64_t total_chunks = g.kh * g.kw * (g.c / acb);
  p.k = static_cast<int32_t>(((total_chunks + 1) / 2) * 128);
  p.ow = static_cast<int32_t>(g.ow);
  p.ohw = static_cast<int32_t>(g.oh * g.ow);
  p.sw = p.sh = 1;
  p.pw = static_cast<int32_t>(g.pw);
  p.ph = static_cast<int32_t>(g.ph);
  p.dw = p.dh = 1;
  p.kw = static_cast<int32_t>(g.kw);
  p.chunks_per_tap = static_cast<int32_t>(g.c / acb);
  p.total_chunks = static_cast<int32_t>(total_chunks);
  fill_outputs(p, bias, scale, s_out, rounding, out_pool, nullptr, nullptr, 256, ds->err_word);
  p.band_rows = static_cast<int32_t>(4 * g.ow);
  p.bands = static_cast<int32_t>(conv_h / 4);
  p.pool_tiles = static_cast<int32_t>(g.n * (conv_h / 4));
  p.conv_w = static_cast<int32_t>(conv_w);
  p.conv_h = static_cast<int32_t>(conv_h);
  p.cout = static_cast<int32_t>(cout);
  p.group = group;
  p.ph_out = static_cast<int32_t>(conv_h / 2);
  p.pw_out = static_cast<int32_t>(conv_w / 2);
  return launch_pool_cfg(ta, tw, p, *ds, stream);
}

}  // namespace lsc

extern "C" lsc_status lsc_debug_withhold_copy(int32_t launches, uint64_t wait_limit_ns) {
  if (launches < 0 || wait_limit_ns < 1000000ull || wait_limit_ns > lsc::kWaitLimitNs)
    return lsc::set_error(LSC_ERROR_INVALID_ARGUMENT,
                          "debug_withhold_copy: launches >= 0 and a wait limit of 1 ms to 2 s");
  lsc::t_withhold.launches = launches;
  lsc::t_withhold.wait_ns = wait_limit_ns;
  return LSC_SUCCESS;
}

extern "C" lsc_status lsc_conv2d_i8_nhwc(const int8_t* x, const int8_t* w, int64_t n, int64_t h,
                                         int64_t wd, int64_t c, int64_t c_out, int64_t kh,
                                         int64_t kw, int64_t sh, int64_t sw, int64_t ph,
                                         int64_t pw, int64_t dh, int64_t dw, const int32_t* bias,
                                         const float* scale, float s_out, int32_t act,
                                         int32_t rounding, int8_t* out_i8, float* out_f32,
                                         int32_t* out_i32, const int8_t* residual,
                                         float residual_scale, lsc_stream stream) {
  lsc::ConvGeometry g{};
  g.n = n;
  g.h = h;
  g.w = wd;
  g.c = c;
  g.c_out = c_out;
  g.kh = kh;
  g.kw = kw;
  g.sh = sh;
  g.sw = sw;
  g.ph = ph;
  g.pw = pw;
  g.dh = dh;
  g.dw = dw;
  g.ph_b = ph;
  g.pw_r = pw;
  if (sh <= 0 || sw <= 0)
    return lsc::set_error(LSC_ERROR_INVALID_ARGUMENT, "conv2d_i8: stride must be positive");
  g.oh = (h + 2 * ph - dh * (kh - 1) - 1) / sh + 1;
  g.ow = (wd + 2 * pw - dw * (kw - 1) - 1) / sw + 1;
  return lsc::launch_conv_i8(x, w, g, bias, scale, s_out, act, rounding, out_i8, out_f32,
                             out_i32, residual, residual_scale, static_cast<cudaStream_t>(stream));
}
