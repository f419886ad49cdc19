// stem_i8.cu -- the ResNet stem of a quantized CNN as one kernel:
//   f32 NCHW [n, 3, 224, 224]
//     -> int8 with the input's per-tensor scale       quantize_value (quantization/helpers.rs:139-155)
//     -> 7x7 / 2 convolution, padding 3, 64 channels   Conv2d::forward (operator/convolution.rs:90-267)
//        + bias, per-channel scale, ReLU, requantize   quantized_ops.rs:36-48, platform/simd.rs:552-556
//     -> 3x3 / 2 max pool, padding 1 (taps skipped)    Pool2d (operator/pooling.rs:383-455)
//   -> int8 NHWC [n, 56, 56, 64]
//
// Separate launches quantize the image into a space-to-depth int8 tensor (HBM round trip),
// convolve it and pool the 205 MB (batch 256) conv output.  Here the input is read once as
// f32, quantized in shared memory, gathered into im2col rows by CUDA cores, contracted on the
// tensor cores (tcgen05 kind::i8, accumulators in TMEM) and pooled on the int32 accumulators:
// the requantization (bias, scale, ReLU, rounding, clamp) is a monotone non-decreasing map of
// the accumulator for a positive channel scale, so the max of the requantized codes over a
// window is the requantized max of the accumulators, and only the pooled quarter of the
// outputs is requantized.  The results are the separate launches' bit for bit.  (The caller --
// the INT8 session's prepare_stem -- checks the conditions that argument needs: positive channel
// scales, and biases small enough that the accumulator plus the bias cannot wrap around:
// |acc| < 147 * 128 * 128 < 2^22.)
//
// One CTA per SM walks a contiguous range of pooled rows (the whole batch's n * 56 rows split
// evenly over the grid).  A pooled row py reads conv rows 2py-1, 2py, 2py+1; consecutive pooled
// rows share the odd conv row, so a CTA computes every conv row of its range once (plus the
// row before its first pooled row).  Warp roles:
//   builders (the 7 warps below 15 with warp % 4 in {2, 3}): one TMA tensor load per conv
//               row brings its two new f32 input rows of the three channels (rows outside the
//               image arrive as zeros), four conv rows ahead; the rows are quantized into a
//               ring of int8 rows held as four copies shifted by 1, 3, 5 and 7 bytes, so that
//               the eight taps (kw = 0..7) of every (channel, kh) pair of an output pixel are
//               one aligned 8-byte load; the conv row's im2col rows (pixel x at row x + 4) go
//               into a B stage (K-major, no swizzle).  Software-pipelined: between two
//               barriers the builders write conv row i's im2col rows and quantize the input
//               rows of conv row i + 1.
//   MMA (warp 15): 6 x tcgen05.mma.cta_group::1.kind::i8 per conv row, M = 128 (the 64 filter
//               rows and 64 zero rows), N = 128 (pixels), K = 32, into one of four 128-column
//               TMEM blocks: TMEM lane = output channel, column = pixel + 4.  Commits free the
//               B stage and publish the block.
//   epilogue (the 8 warps with warp % 4 in {0, 1}): lane quarter q holds
//               channels 32q .. 32q + 31, warp w / 4 a quarter of the pooled columns.  Per pooled
//               row each thread loads its channel's 32 columns of the three conv rows, takes the
//               vertical max, releases the blocks no later row needs, then the horizontal
//               windows in registers, bias, scale, ReLU, requantization and byte stores (a
//               warp's 32 channels of one pixel: one 32-byte sector).
// K order of the filter: k = 8 * (c * 7 + kh) + kw for kw in 0..7 (kw = 7 has zero weight),
// 168 taps padded to 192 with zeros.
// Every mbarrier wait is bounded (sm100.cuh); a wait that runs out sets the error word, the
// CTA's abort flag makes the other roles leave, and TMEM is freed before the CTA exits.
#include <math.h>

#include <cmath>
#include <cstring>
#include <mutex>

#include "epilogue.cuh"
#include "lsc_internal.h"
#include "sm100.cuh"

namespace lsc {
namespace {

constexpr int kStH = 224, kStW = 224, kStC = 3;
constexpr int kStOW = 112;              // conv output width (and height)
constexpr int kStPH = 56, kStPW = 56;   // pool output
constexpr int kStCout = 64;
constexpr int kStK = 192;               // 21 (c, kh) groups x 8 taps = 168, padded to 6 x 32
constexpr int kStKSteps = kStK / 32;
constexpr int kStStages = 3;
constexpr int kStABytes = (kStK / 16) * 128 * 16;   // 12 chunks of [128 rows][16 B] (filter, im2col)
constexpr int kStF32Slots = 12;    // TMA loads of two f32 input rows x 3 channels
constexpr int kStF32Load = 2 * kStC * kStW * 4;     // bytes per load: [c][2 rows][224]
constexpr int kStRingRows = 16;     // quantized input rows, by a running row count
constexpr int kStCopyPitch = 288;   // one shifted copy of a quantized row (bank-spread)
constexpr int kStLead = 4;          // conv rows whose input is fetched ahead
constexpr int kStBuilders = 224;  // 7 warps: two threads per im2col row of the 112 pixels
constexpr int kStMmaWarp = 15;
constexpr int kStEpiWarps = 8;
constexpr int kStThreads = (kStMmaWarp + 1) * 32;
constexpr int kStTmemBlocks = 4;
constexpr int kStTmemCols = 512;    // four 128-column accumulator blocks

constexpr int kOffW = 0;
constexpr int kOffA = kOffW + kStABytes;
constexpr int kOffF32 = kOffA + kStStages * kStABytes;
constexpr int kOffRing = kOffF32 + kStF32Slots * kStF32Load;
constexpr int kOffBar = kOffRing + kStRingRows * kStC * 4 * kStCopyPitch;
constexpr int kStSmem = kOffBar + 32 * 8 + 1024;  // + alignment of the dynamic base
static_assert(kOffA % 1024 == 0 && kOffF32 % 128 == 0 && kStF32Load % 128 == 0 && kOffRing % 16 == 0 && kOffBar % 8 == 0, "alignment");
static_assert(kStSmem <= 232448, "shared memory");

struct StemParams {
  int8_t* out;
  const int8_t* w;  // the filter's shared-memory image (stem_filter_image)
  const int32_t* bias;
  const float* scale;
  float s_in, inv_s_in;    // input quantization
  float s_out, inv_s_out;  // conv output requantization (inv_s_out 0: division everywhere)
  int32_t rounding;        // of the conv output
  int32_t n;
  uint32_t* err;
};

// Conv row i of a CTA's sequence: image n, row r; `first` when no earlier row of the same
// image precedes it in the sequence (all seven input rows of its window are new).  e = 1 when
// the CTA's first pooled row has py > 0: its upper window row 2py - 1 leads the sequence.
struct StemItem {
  int n, r, first;
};
__device__ __forceinline__ StemItem stem_item(int i, int g0, int e) {
  StemItem it;
  if (e && i == 0) {
    it.n = g0 / kStPH;
    it.r = 2 * (g0 - it.n * kStPH) - 1;
    it.first = 1;
    return it;
  }
  const int j = i - e;
  const int g = g0 + (j >> 1);
  it.n = g / kStPH;
  it.r = 2 * (g - it.n * kStPH) + (j & 1);
  it.first = (i == 0 || it.r == 0) ? 1 : 0;
  return it;
}
// TMA loads of two input rows that conv row `it` needs beyond the previous row of the
// sequence: rows 2r-3 .. 2r+4 (four loads, the last row unused) for a first row, else rows
// 2r+2, 2r+3; and the input rows it adds to the quantized ring (7 or 2)
__device__ __forceinline__ int stem_loads(const StemItem& it) { return it.first ? 4 : 1; }
__device__ __forceinline__ int stem_new_rows(const StemItem& it) { return it.first ? 7 : 2; }
__device__ __forceinline__ int stem_first_row(const StemItem& it) { return it.first ? 2 * it.r - 3 : 2 * it.r + 2; }

template <int RND_IN>
__global__ void __launch_bounds__(kStThreads, 1)
    stem_conv_pool_kernel(const __grid_constant__ CUtensorMap tmX, const StemParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sW = smem + kOffW;
  uint8_t* sA = smem + kOffA;
  uint8_t* f32r = smem + kOffF32;
  uint8_t* ring = smem + kOffRing;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* afull = bars;                  // [kStStages] B stage written (7 builder warps)
  uint64_t* aempty = bars + kStStages;     // [kStStages] B stage read by the MMAs
  uint64_t* tfull = bars + 2 * kStStages;  // [4] TMEM block holds a finished conv row
  uint64_t* tempty = tfull + kStTmemBlocks;  // [4] TMEM block released (8 epilogue warps)
  uint64_t* drain = tempty + kStTmemBlocks;
  uint64_t* xfull = drain + 1;               // [kStF32Slots] input load landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(xfull + kStF32Slots);
  volatile uint32_t* abort_flag = tmem_slot + 1;
  volatile uint32_t* build_ok = tmem_slot + 2;  // the builders' shared verdict on a stage wait

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t G = static_cast<int64_t>(p.n) * kStPH;
  const int g0 = static_cast<int>((static_cast<int64_t>(blockIdx.x) * G) / gridDim.x);
  const int g1 = static_cast<int>((static_cast<int64_t>(blockIdx.x + 1) * G) / gridDim.x);
  const int e = (g0 % kStPH) != 0 ? 1 : 0;
  const int items = 2 * (g1 - g0) + e;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStStages; ++s) {
      mbar_init(&afull[s], kStBuilders / 32);
      mbar_init(&aempty[s], 1);
    }
    for (int b = 0; b < kStTmemBlocks; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], kStEpiWarps);
    }
    mbar_init(drain, 1);
    for (int f = 0; f < kStF32Slots; ++f) mbar_init(&xfull[f], 1);
    *abort_flag = 0u;
    *build_ok = 1u;
    fence_barrier_init();
  }
  if (warp == kStMmaWarp) {
    tmem_alloc(tmem_slot, kStTmemCols);
    tmem_relinquish();
  }
  if (threadIdx.x == 0) tma_prefetch_desc(&tmX);
  // constant operands before the wait for the previous kernel: the filter as the A operand
  // (image rows 0-63, K chunks 1024 bytes apart, moved to 2048; rows 64-127 zero), and the B
  // stages' last K chunk (taps 176..191: zero weights; the builders never write it)
  for (int i = threadIdx.x; i < 12 * 128; i += blockDim.x) {
    const int chunk = i >> 7, row = i & 127;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (row < kStCout) v = __ldg(reinterpret_cast<const uint4*>(p.w + chunk * 1024 + row * 16));
    *reinterpret_cast<uint4*>(sW + chunk * 2048 + row * 16) = v;
  }
  for (int i = threadIdx.x; i < kStStages * 128; i += blockDim.x)
    *reinterpret_cast<uint4*>(sA + (i >> 7) * kStABytes + 11 * 2048 + (i & 127) * 16) = make_uint4(0u, 0u, 0u, 0u);
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  griddep_wait();  // the input and the output belong to earlier work until it completes
  griddep_launch_dependents();

  if (warp < kStMmaWarp && (warp & 3) >= 2) {
    // ------------------------------------------------------------------ builders
    const int bwarp = (warp >> 2) * 2 + (warp & 1);  // 0..6
    const int t = bwarp * 32 + lane;
    // input loads in sequence order: slot = count mod kStF32Slots.  Thread 0 issues the loads
    // of conv row i + kStLead + 1 after the barrier of iteration i, when every builder has
    // quantized row i's input; rows i+1 .. i+5 then hold at most 4 + 1 + 1 + 4 + 1 loads (first
    // rows are at least three rows apart), within the twelve slots.
    int issued_item = 0, issued_loads = 0;  // thread 0
    auto issue_upto = [&](int upto) {
      for (; issued_item <= upto && issued_item < items; ++issued_item) {
        const StemItem it = stem_item(issued_item, g0, e);
        const int y0 = stem_first_row(it);
        for (int j = 0; j < stem_loads(it); ++j, ++issued_loads) {
          const int slot = issued_loads % kStF32Slots;
          mbar_arrive_expect_tx(&xfull[slot], kStF32Load);
          tma_load_4d(&tmX, &xfull[slot], f32r + slot * kStF32Load, 0, y0 + 2 * j, 0, it.n);
        }
      }
    };
    int used_loads = 0;  // loads consumed (all builders)
    int qrows = 0;       // input rows quantized into the ring (all builders)
    bool ok = true;
    // quantize the new input rows of conv row k: one (row, channel) per warp; lane l quantizes
    // words l and l + 32 of the row image P (word u = columns 4u-8 .. 4u-5, P[i] = q(x[i - 8]),
    // zero outside the image), then writes words l and l + 32 (< 62) of the copies shifted by
    // 1, 3, 5 and 7 bytes into ring row qrows mod 16, the next two words from lanes l+1, l+2
    auto quantize = [&](int k) -> bool {
      const StemItem it = stem_item(k, g0, e);
      const int nl = stem_loads(it), nr = stem_new_rows(it);
      for (int j = 0; j < nl; ++j) {
        const int u = used_loads + j;
        if (!mbar_wait(&xfull[u % kStF32Slots], (u / kStF32Slots) & 1, abort_flag, p.err)) return false;
      }
#pragma unroll 1
      for (int task = bwarp; task < nr * kStC; task += kStBuilders / 32) {
        const int ri = task / kStC, c = task - ri * kStC;
        const float* row = reinterpret_cast<const float*>(
            f32r + ((used_loads + (ri >> 1)) % kStF32Slots) * kStF32Load + (c * 2 + (ri & 1)) * (kStW * 4));
        uint32_t pw[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int u = lane + 32 * h;
          float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
          if (u >= 2 && u <= 57) {
            const float4 f = *reinterpret_cast<const float4*>(row + 4 * u - 8);
            v[0] = f.x;
            v[1] = f.y;
            v[2] = f.z;
            v[3] = f.w;
          }
          uint32_t pk[1];
          requant_pack_rnd<4, RND_IN>(v, p.s_in, p.inv_s_in, false, pk);
          pw[h] = pk[0];
        }
        const int l1 = (lane + 1) & 31, l2 = (lane + 2) & 31;
        const uint32_t a1_0 = __shfl_sync(0xFFFFFFFFu, pw[0], l1), a1_1 = __shfl_sync(0xFFFFFFFFu, pw[1], l1);
        const uint32_t a2_0 = __shfl_sync(0xFFFFFFFFu, pw[0], l2), a2_1 = __shfl_sync(0xFFFFFFFFu, pw[1], l2);
        uint8_t* dst = ring + (((qrows + ri) & (kStRingRows - 1)) * kStC + c) * 4 * kStCopyPitch + 4 * lane;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          if (h == 1 && lane >= 30) break;  // words 62, 63 of the copies are never read
          const uint32_t a = pw[h];
          const uint32_t b = h == 0 ? (lane < 31 ? a1_0 : a1_1) : a1_1;
          const uint32_t d = h == 0 ? (lane < 30 ? a2_0 : a2_1) : a2_1;
          uint8_t* o = dst + 128 * h;
          *reinterpret_cast<uint32_t*>(o) = __funnelshift_r(a, b, 8);
          *reinterpret_cast<uint32_t*>(o + kStCopyPitch) = __funnelshift_r(a, b, 24);
          *reinterpret_cast<uint32_t*>(o + 2 * kStCopyPitch) = __funnelshift_r(b, d, 8);
          *reinterpret_cast<uint32_t*>(o + 3 * kStCopyPitch) = __funnelshift_r(b, d, 24);
        }
      }
      used_loads += nl;
      qrows += nr;
      return true;
    };
    if (t == 0) issue_upto(kStLead);
    ok = quantize(0);
#pragma unroll 1
    for (int i = 0; i < items; ++i) {
      const int s = i % kStStages;
      if (t == 0) {
        if (!ok || !mbar_wait(&aempty[s], ((i / kStStages) & 1) ^ 1u, abort_flag, p.err)) *build_ok = 0u;
      }
      if (!ok) *build_ok = 0u;  // a builder whose input wait ran out
      named_bar_sync(1, kStBuilders);
      if (!*build_ok) break;
      if (t == 0) issue_upto(i + kStLead + 1);
      // the im2col row of output pixel x at B row x + 4 (rows 0-3 and 116-127 are never read
      // back) from the last seven quantized rows (input rows 2r-3 .. 2r+3); threads 0-111 write
      // K chunks 0-5 ((c, kh) groups 0-11) of pixels 0-111, threads 112-223 chunks 6-10
      {
        const int nrow = 4 + (t < kStOW ? t : t - kStOW);
        const int o = 2 * (nrow - 4) + 5;  // P index of input column 2x - 3
        const uint8_t* rb = ring + ((o & 7) >> 1) * kStCopyPitch + (o & ~7);
        uint8_t* ab = sA + s * kStABytes + nrow * 16;
        const int row0 = qrows - 7;  // ring rows of conv row i (row i + 1's come after the build)
        auto group = [&](int q) -> uint2 {
          const int c = q / 7, kh = q - 7 * (q / 7);
          const int slot = (row0 + kh) & (kStRingRows - 1);
          return *reinterpret_cast<const uint2*>(rb + (slot * kStC + c) * 4 * kStCopyPitch);
        };
        if (t < kStOW) {
          uint2 v[12];
#pragma unroll
          for (int q = 0; q < 12; ++q) v[q] = group(q);
#pragma unroll
          for (int j = 0; j < 6; ++j)
            *reinterpret_cast<uint4*>(ab + j * 2048) = make_uint4(v[2 * j].x, v[2 * j].y, v[2 * j + 1].x, v[2 * j + 1].y);
        } else {
          uint2 v[9];
#pragma unroll
          for (int q = 0; q < 9; ++q) v[q] = group(12 + q);
#pragma unroll
          for (int j = 0; j < 4; ++j)
            *reinterpret_cast<uint4*>(ab + (6 + j) * 2048) =
                make_uint4(v[2 * j].x, v[2 * j].y, v[2 * j + 1].x, v[2 * j + 1].y);
          *reinterpret_cast<uint4*>(ab + 10 * 2048) = make_uint4(v[8].x, v[8].y, 0u, 0u);
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&afull[s]);
      if (i + 1 < items) ok = quantize(i + 1);
    }
    if (t == 0) {  // loads still in flight land before the CTA exits
      volatile uint32_t no_abort = 0u;
      for (int u = used_loads; u < issued_loads; ++u)
        mbar_wait(&xfull[u % kStF32Slots], (u / kStF32Slots) & 1, &no_abort, p.err);
    }
  } else if (warp == kStMmaWarp) {
    // ------------------------------------------------------------------ MMA issuer
    constexpr uint32_t idesc = idesc_i8(128, 128);
    uint64_t adesc[kStKSteps], bdesc[kStKSteps];
#pragma unroll
    for (int kk = 0; kk < kStKSteps; ++kk) {
      adesc[kk] = smem_desc_noswz_kmajor(smem_u32(sW) + kk * 2 * 2048, 2048, 128);
      bdesc[kk] = smem_desc_noswz_kmajor(smem_u32(sA) + kk * 2 * 2048, 2048, 128);
    }
    bool ok = true, any = false;
#pragma unroll 1
    for (int i = 0; i < items && ok; ++i) {
      const int b = i & (kStTmemBlocks - 1), s = i % kStStages;
      ok = __all_sync(0xFFFFFFFFu, mbar_wait(&tempty[b], ((i / kStTmemBlocks) & 1) ^ 1u, abort_flag, p.err));
      if (!ok) break;
      ok = __all_sync(0xFFFFFFFFu, mbar_wait(&afull[s], (i / kStStages) & 1, abort_flag, p.err));
      if (!ok) break;
      tc_fence_after();
      if (elect_one()) {
        const uint64_t bo = static_cast<uint64_t>(s * (kStABytes >> 4));
        const uint32_t d = tmem_base + static_cast<uint32_t>(b * 128);
#pragma unroll
        for (int kk = 0; kk < kStKSteps; ++kk) mma_i8(d, adesc[kk], bdesc[kk] + bo, idesc, kk != 0 ? 1u : 0u);
        mma_commit(&aempty[s]);
        mma_commit(&tfull[b]);
      }
      __syncwarp();
      any = true;
    }
    if (!ok && any) {  // MMAs in flight must finish before TMEM is released
      if (elect_one()) mma_commit(drain);
      __syncwarp();
      volatile uint32_t no_abort = 0u;
      mbar_wait(drain, 0u, &no_abort, p.err);
    }
  } else if (warp < kStMmaWarp) {
    // ------------------------------------------------------------------ epilogue
    const int quarter = warp & 3;           // 0 or 1: TMEM lanes = channels 32q .. 32q + 31
    const int slice = warp >> 2;            // pooled columns 14 * slice .. 14 * slice + 13
    const int ch = quarter * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    // this thread's conv columns: x = 28 * slice - 4 + i at TMEM column 28 * slice + i
    const uint32_t col0 = static_cast<uint32_t>(28 * slice);
    const int32_t bias = p.bias ? __ldg(p.bias + ch) : 0;
    const float scale = __ldg(p.scale + ch);
    const bool relu_folded = p.inv_s_out > 0.0f;
    int rel = 0;
    bool ok = true;
#pragma unroll 1
    for (int gi = g0; gi < g1; ++gi) {
      const int n = gi / kStPH, py = gi - n * kStPH;
      const int il = e + 2 * (gi - g0) + 1;  // conv row 2py + 1; 2py and 2py - 1 precede it
      bool w = mbar_wait(&tfull[il & 3], (il >> 2) & 1, abort_flag, p.err);
      w = w && mbar_wait(&tfull[(il - 1) & 3], ((il - 1) >> 2) & 1, abort_flag, p.err);
      if (py > 0) w = w && mbar_wait(&tfull[(il - 2) & 3], ((il - 2) >> 2) & 1, abort_flag, p.err);
      ok = __all_sync(0xFFFFFFFFu, w);
      if (!ok) break;
      tc_fence_after();
      // vertical window: max of conv rows 2py - 1 (absent at py = 0), 2py, 2py + 1
      int32_t m[32];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t ra[16], rb[16], rc[16];
        const uint32_t cofs = lane_off + col0 + 16u * h;
        tmem_ld_32x32b_x16(tmem_base + cofs + static_cast<uint32_t>((il & 3) * 128), ra);
        tmem_ld_32x32b_x16(tmem_base + cofs + static_cast<uint32_t>(((il - 1) & 3) * 128), rb);
        if (py > 0) tmem_ld_32x32b_x16(tmem_base + cofs + static_cast<uint32_t>(((il - 2) & 3) * 128), rc);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 16; ++j)
          m[16 * h + j] = py > 0 ? __vimax3_s32(static_cast<int32_t>(ra[j]), static_cast<int32_t>(rb[j]),
                                                static_cast<int32_t>(rc[j]))
                                 : max(static_cast<int32_t>(ra[j]), static_cast<int32_t>(rb[j]));
      }
      // release the conv rows no later pooled row reads (the odd row 2py + 1 stays for the
      // next pooled row of the same image): the MMAs refill them while this row finishes
      const int target = (gi + 1 == g1 || py == kStPH - 1) ? il + 1 : il;
      tc_fence_before();
      __syncwarp();
      for (; rel < target; ++rel)
        if (lane == 0) mbar_arrive(&tempty[rel & 3]);
      // horizontal windows: pooled column 14 * slice + j reads conv columns 2j + 3 .. 2j + 5
      // of m (x = 28 * slice + 2j - 1 .. + 1); at pooled column 0 the left tap is padding
      float y[16];
#pragma unroll
      for (int j = 0; j < 14; j += 2) {
        int32_t v0 = __vimax3_s32(m[2 * j + 3], m[2 * j + 4], m[2 * j + 5]);
        if (j == 0 && slice == 0) v0 = max(m[4], m[5]);
        const int32_t v1 = __vimax3_s32(m[2 * j + 5], m[2 * j + 6], m[2 * j + 7]);
        const int32_t a0 = static_cast<int32_t>(static_cast<uint32_t>(v0) + static_cast<uint32_t>(bias));
        const int32_t a1 = static_cast<int32_t>(static_cast<uint32_t>(v1) + static_cast<uint32_t>(bias));
        f2unpack(f2mul(f2pack(__int2float_rn(a0), __int2float_rn(a1)), f2pack(scale, scale)), y[j], y[j + 1]);
      }
      y[14] = 0.0f;
      y[15] = 0.0f;
      if (!relu_folded) {
#pragma unroll
        for (int j = 0; j < 14; ++j) y[j] = apply_act<LSC_ACT_RELU>(y[j]);
      }
      uint32_t pk[4];
      requant_pack<16>(y, p.s_out, p.inv_s_out, relu_folded, p.rounding, pk);
      int8_t* dst = p.out + ((static_cast<int64_t>(n) * kStPH + py) * kStPW + 14 * slice) * kStCout + ch;
#pragma unroll
      for (int j = 0; j < 14; ++j) dst[j * kStCout] = static_cast<int8_t>(pk[j >> 2] >> (8 * (j & 3)));
    }
  }

  __syncthreads();
  if (warp == kStMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kStTmemCols);
  }
}

}  // namespace

void stem_filter_image(const int8_t* w_s2d, int8_t* img) {
  std::memset(img, 0, static_cast<size_t>(kStemFilterBytes));
  for (int co = 0; co < kStCout; ++co)
    for (int c = 0; c < kStC; ++c)
      for (int kh = 0; kh < 7; ++kh)
        for (int kw = 0; kw < 7; ++kw) {
          // space-to-depth filter [co][kh / 2][kw / 2][((kh % 2) * 2 + kw % 2) * 3 + c], 16 channels
          const int8_t v = w_s2d[((co * 4 + kh / 2) * 4 + kw / 2) * 16 + ((kh % 2) * 2 + kw % 2) * 3 + c];
          const int k = 8 * (c * 7 + kh) + kw;
          img[(k / 16) * 1024 + (co / 8) * 128 + (co % 8) * 16 + (k % 16)] = v;
        }
}

lsc_status launch_stem_conv_pool_i8(const float* x, int64_t n, const int8_t* w_img, const int32_t* bias,
                                    const float* scale, float s_in, int rounding_in, float s_out, int rounding,
                                    int8_t* out, cudaStream_t stream) {
  if (!x || !w_img || !scale || !out)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "stem_conv_pool_i8: null pointer");
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w_img) | reinterpret_cast<uintptr_t>(out)) & 15)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "stem_conv_pool_i8: x, the filter and the output must be 16-byte aligned");
  if (n <= 0 || n * kStPH > INT32_MAX / 2)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "stem_conv_pool_i8: batch out of range");
  if ((rounding != LSC_ROUND_HALF_AWAY && rounding != LSC_ROUND_HALF_EVEN) ||
      (rounding_in != LSC_ROUND_HALF_AWAY && rounding_in != LSC_ROUND_HALF_EVEN))
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "stem_conv_pool_i8: unknown rounding mode");
  if (!(s_out > 0.0f) || !std::isfinite(s_out))
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "stem_conv_pool_i8: the output scale must be positive");
  DeviceState* ds = current_device_state();
  if (!ds) return LSC_ERROR_DEVICE_ERROR;
  if (ds->cc_major != 10) return set_error(LSC_ERROR_BACKEND_NOT_AVAILABLE, "stem_conv_pool_i8: needs an sm_100 (B200) device");
  auto kernel = rounding_in == LSC_ROUND_HALF_EVEN ? stem_conv_pool_kernel<LSC_ROUND_HALF_EVEN>
                                                   : stem_conv_pool_kernel<LSC_ROUND_HALF_AWAY>;
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [] {
    attr_err = cudaFuncSetAttribute(stem_conv_pool_kernel<LSC_ROUND_HALF_EVEN>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, kStSmem);
    if (attr_err == cudaSuccess)
      attr_err = cudaFuncSetAttribute(stem_conv_pool_kernel<LSC_ROUND_HALF_AWAY>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, kStSmem);
  });
  if (attr_err != cudaSuccess) return cuda_error(attr_err, "cudaFuncSetAttribute(stem_conv_pool)");
  CUtensorMap tmx;
  const uint64_t dims[4] = {static_cast<uint64_t>(kStW), static_cast<uint64_t>(kStH), static_cast<uint64_t>(kStC),
                            static_cast<uint64_t>(n)};
  const uint64_t strides[3] = {static_cast<uint64_t>(kStW) * 4, static_cast<uint64_t>(kStH) * kStW * 4,
                               static_cast<uint64_t>(kStC) * kStH * kStW * 4};
  const uint32_t box[4] = {static_cast<uint32_t>(kStW), 2u, static_cast<uint32_t>(kStC), 1u};
  const uint32_t estr[4] = {1u, 1u, 1u, 1u};
  lsc_status st = encode_tmap_4d(&tmx, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, x, dims, strides, box, estr,
                                 CU_TENSOR_MAP_SWIZZLE_NONE);
  if (st) return st;
  StemParams p{};
  p.out = out;
  p.w = w_img;
  p.bias = bias;
  p.scale = scale;
  p.s_in = s_in;
  p.inv_s_in = reciprocal_or_zero(s_in);
  p.s_out = s_out;
  const float inv = 1.0f / s_out;
  p.inv_s_out = (std::isnormal(s_out) && std::isnormal(inv)) ? inv : 0.0f;
  p.rounding = rounding;
  p.n = static_cast<int32_t>(n);
  p.err = ds->err_word;
  const int64_t rows = n * kStPH;
  const int grid = static_cast<int>(rows < ds->sm_count ? rows : ds->sm_count);
  LSC_CUDA_TRY(launch_dependent(ds->overlap_launches, kernel, dim3(grid), dim3(kStThreads), static_cast<size_t>(kStSmem),
                                stream, tmx, p));
  return LSC_SUCCESS;
}

}  // namespace lsc
