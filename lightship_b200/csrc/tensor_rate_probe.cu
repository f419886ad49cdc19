// tensor_rate_probe.cu -- the tensor pipe's issue rate on resident shared-memory operands.
//
// The ceiling every contraction kernel here is measured against: one thread per CTA issues
// `iters` back-to-back tcgen05.mma instructions over operands that never leave shared memory
// (no TMA, no epilogue, no barrier round trip between instructions), commits once and waits
// for completion; clock64 and %globaltimer around the sequence give cycles and nanoseconds per
// instruction.  Run on one CTA per SM across the whole GPU it also shows the clock the tensor
// pipe sustains under load.  Shapes: M = 128 (cta_group::1) or 256 (cta_group::2, a CTA pair),
// N = 64 / 128 / 256, K = 32 bytes (kind::i8: 32 int8 values; kind::f16: 16 f16 values), 128-byte
// swizzled K-major operands as the contraction kernels lay them out.  The operands are zero:
// the values do not change the issue rate.
#include <algorithm>
#include <vector>

#include "lsc_internal.h"
#include "sm100.cuh"

namespace lsc {
namespace {

constexpr int kProbeThreads = 128;
constexpr int kProbeABytes = 128 * 128;
constexpr int kProbeBBytes = 256 * 128;
constexpr int kProbeSmem = kProbeABytes + kProbeBBytes + 1024 + 128;

__device__ __forceinline__ void mma_f16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// KIND 0: kind::i8 (s32 accumulators), 1: kind::f16 (f32 accumulators).  PAIR: clusters of two
// CTAs, the even one issuing M = 256 instructions over both CTAs' shared memory.
// The issue loop's shape (MODE) is the variable under study:
//   0  one flat loop of instructions, nothing else in it;
//   1  the flat loop with a runtime-optional commit (every `commit_every` instructions, onto
//      one of eight mbarriers in turn) and a bounded wait for the commit `wait_lag` back;
//   2  k-blocks of four instructions (unrolled), a commit after each k-block and, with
//      wait_lag > 0, a bounded wait for the commit wait_lag k-blocks back -- the cadence of a
//      pipelined kernel's stage releases, without its loads;
//   3  as 2, the whole warp running the loop and one elected lane issuing (warp converged);
//   4  as 2 with the wait a test_wait spin (never suspends; bounded by a spin count).
template <int KIND, int N, bool PAIR>
__device__ __forceinline__ void probe_mma(uint32_t d_tmem, uint64_t ad, uint64_t bd, uint32_t acc) {
  constexpr uint32_t M = PAIR ? 256 : 128;
  constexpr uint32_t IDESC = KIND == 0 ? idesc_i8(M, N) : idesc_f16(M, N);
  if constexpr (PAIR) {
    if constexpr (KIND == 0) mma_i8_pair(d_tmem, ad, bd, IDESC, acc);
    else mma_f16_pair(d_tmem, ad, bd, IDESC, acc);
  } else {
    if constexpr (KIND == 0) mma_i8(d_tmem, ad, bd, IDESC, acc);
    else mma_f16(d_tmem, ad, bd, IDESC, acc);
  }
}

template <bool PAIR>
__device__ __forceinline__ void probe_commit(uint64_t* bar) {
  if constexpr (PAIR) mma_commit_pair(bar, 0x1);
  else mma_commit(bar);
}

// A wait that never suspends the thread: test_wait in a loop bounded by a count.
__device__ __forceinline__ bool spin_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t a = smem_u32(bar);
  for (uint32_t i = 0; i < (1u << 28); ++i)
    if (mbar_test_wait(a, parity)) return true;
  return false;
}

template <int KIND, int N, bool PAIR, int MODE>
__global__ void __launch_bounds__(kProbeThreads, 1)
    tensor_rate_probe_kernel(int iters, int commit_every, int wait_lag, unsigned long long* cycles,
                             unsigned long long* nanos, uint32_t* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + kProbeABytes;
  uint64_t* done = reinterpret_cast<uint64_t*>(sB + kProbeBBytes);
  uint64_t* ring = done + 1;  // 8 stage-release barriers
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ring + 8);
  volatile uint32_t* abort_flag = tmem_slot + 1;
  constexpr uint32_t kCols = N < 32 ? 32 : N;
  const int warp = threadIdx.x >> 5;
  uint32_t rank = 0;
  if constexpr (PAIR) rank = cluster_ctarank();

  for (int i = threadIdx.x; i < (kProbeABytes + kProbeBBytes) / 16; i += blockDim.x)
    reinterpret_cast<uint4*>(smem)[i] = make_uint4(0u, 0u, 0u, 0u);
  fence_proxy_async_smem();
  if (threadIdx.x == 0) {
    mbar_init(done, 1);
    for (int i = 0; i < 8; ++i) mbar_init(&ring[i], 1);
    *abort_flag = 0u;
    fence_barrier_init();
  }
  if (warp == 0) {
    if constexpr (PAIR) {
      tmem_alloc_pair(tmem_slot, kCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, kCols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync();
  tc_fence_after();
  const uint32_t d_tmem = *tmem_slot;
  const uint32_t a0 = smem_u32(sA), b0 = smem_u32(sB);
  const bool issuer_cta = rank == 0;

  if constexpr (MODE == 3) {
    if (warp == 0 && issuer_cta) {
      const unsigned long long g0 = globaltimer_ns();
      const long long c0 = clock64();
      bool ok = true;
      const int kblocks = iters / 4;
      for (int kb = 0; kb < kblocks && ok; ++kb) {
        if (elect_one()) {
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            probe_mma<KIND, N, PAIR>(d_tmem, smem_desc_sw128_kmajor(a0 + kk * 32),
                                     smem_desc_sw128_kmajor(b0 + kk * 32), (kb | kk) != 0 ? 1u : 0u);
          probe_commit<PAIR>(&ring[kb & 7]);
        }
        __syncwarp();
        if (wait_lag > 0 && kb >= wait_lag) {
          const int c = kb - wait_lag;
          ok = mbar_wait(&ring[c & 7], static_cast<uint32_t>((c >> 3) & 1), abort_flag, err);
        }
      }
      if (elect_one()) probe_commit<PAIR>(done);
      __syncwarp();
      ok = mbar_wait(done, 0u, abort_flag, err) && ok;
      const long long c1 = clock64();
      const unsigned long long g1 = globaltimer_ns();
      if (threadIdx.x == 0) {
        const int slot = PAIR ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
        cycles[slot] = ok ? static_cast<unsigned long long>(c1 - c0) : 0ull;
        nanos[slot] = ok ? g1 - g0 : 0ull;
      }
    }
  } else if (threadIdx.x == 0 && issuer_cta) {
    const unsigned long long g0 = globaltimer_ns();
    const long long c0 = clock64();
    bool ok = true;
    if constexpr (MODE == 0) {
      for (int i = 0; i < iters; ++i) {
        const uint32_t kk = static_cast<uint32_t>(i & 3) * 32u;
        probe_mma<KIND, N, PAIR>(d_tmem, smem_desc_sw128_kmajor(a0 + kk), smem_desc_sw128_kmajor(b0 + kk),
                                 i != 0 ? 1u : 0u);
      }
    } else if constexpr (MODE == 1) {
      int commits = 0;
      for (int i = 0; i < iters && ok; ++i) {
        const uint32_t kk = static_cast<uint32_t>(i & 3) * 32u;
        probe_mma<KIND, N, PAIR>(d_tmem, smem_desc_sw128_kmajor(a0 + kk), smem_desc_sw128_kmajor(b0 + kk),
                                 i != 0 ? 1u : 0u);
        if (commit_every > 0 && (i + 1) % commit_every == 0) {
          probe_commit<PAIR>(&ring[commits & 7]);
          ++commits;
          if (wait_lag > 0 && commits > wait_lag) {
            const int c = commits - 1 - wait_lag;
            ok = mbar_wait(&ring[c & 7], static_cast<uint32_t>((c >> 3) & 1), abort_flag, err);
          }
        }
      }
    } else {
      const int kblocks = iters / 4;
      for (int kb = 0; kb < kblocks && ok; ++kb) {
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          probe_mma<KIND, N, PAIR>(d_tmem, smem_desc_sw128_kmajor(a0 + kk * 32), smem_desc_sw128_kmajor(b0 + kk * 32),
                                   (kb | kk) != 0 ? 1u : 0u);
        probe_commit<PAIR>(&ring[kb & 7]);
        if (wait_lag > 0 && kb >= wait_lag) {
          const int c = kb - wait_lag;
          const uint32_t par = static_cast<uint32_t>((c >> 3) & 1);
          if constexpr (MODE == 2) ok = mbar_wait(&ring[c & 7], par, abort_flag, err);
          else ok = spin_wait(&ring[c & 7], par);
        }
      }
    }
    probe_commit<PAIR>(done);
    ok = mbar_wait(done, 0u, abort_flag, err) && ok;
    const long long c1 = clock64();
    const unsigned long long g1 = globaltimer_ns();
    const int slot = PAIR ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
    cycles[slot] = ok ? static_cast<unsigned long long>(c1 - c0) : 0ull;
    nanos[slot] = ok ? g1 - g0 : 0ull;
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync();
  if (warp == 0) {
    tc_fence_after();
    if constexpr (PAIR) tmem_dealloc_pair(d_tmem, kCols);
    else tmem_dealloc(d_tmem, kCols);
  }
}

template <int KIND, int N, bool PAIR, int MODE>
lsc_status run_probe(int iters, int commit_every, int wait_lag, int ctas, unsigned long long* cycles,
                     unsigned long long* nanos, uint32_t* err) {
  auto kernel = tensor_rate_probe_kernel<KIND, N, PAIR, MODE>;
  LSC_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kProbeSmem));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(PAIR ? 2 * ctas : ctas);
  cfg.blockDim = dim3(kProbeThreads);
  cfg.dynamicSmemBytes = kProbeSmem;
  cudaLaunchAttribute attr[1];
  if (PAIR) {
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  LSC_CUDA_TRY(cudaLaunchKernelEx(&cfg, kernel, iters, commit_every, wait_lag, cycles, nanos, err));
  return LSC_SUCCESS;
}

template <int KIND, bool PAIR, int MODE>
lsc_status run_probe_n(int n, int iters, int ce, int lag, int ctas, unsigned long long* cycles,
                       unsigned long long* nanos, uint32_t* err) {
  switch (n) {
    case 64: return run_probe<KIND, 64, PAIR, MODE>(iters, ce, lag, ctas, cycles, nanos, err);
    case 128: return run_probe<KIND, 128, PAIR, MODE>(iters, ce, lag, ctas, cycles, nanos, err);
    case 256: return run_probe<KIND, 256, PAIR, MODE>(iters, ce, lag, ctas, cycles, nanos, err);
    default: return set_error(LSC_ERROR_INVALID_ARGUMENT, "probe_tensor_rate: N must be 64, 128 or 256");
  }
}

template <int KIND, bool PAIR>
lsc_status run_probe_mode(int mode, int n, int iters, int ce, int lag, int ctas, unsigned long long* cycles,
                          unsigned long long* nanos, uint32_t* err) {
  switch (mode) {
    case 0: return run_probe_n<KIND, PAIR, 0>(n, iters, ce, lag, ctas, cycles, nanos, err);
    case 1: return run_probe_n<KIND, PAIR, 1>(n, iters, ce, lag, ctas, cycles, nanos, err);
    case 2: return run_probe_n<KIND, PAIR, 2>(n, iters, ce, lag, ctas, cycles, nanos, err);
    case 3: return run_probe_n<KIND, PAIR, 3>(n, iters, ce, lag, ctas, cycles, nanos, err);
    case 4: return run_probe_n<KIND, PAIR, 4>(n, iters, ce, lag, ctas, cycles, nanos, err);
    default: return set_error(LSC_ERROR_INVALID_ARGUMENT, "probe_tensor_rate: mode 0..4");
  }
}

// ---------------------------------------------------------------------------------------
// Operand delivery: how many bytes per clock one SM's TMA unit brings from L2 into shared
// memory.  `warps` producer threads (lane 0 of each warp) each keep `depth` tile loads in
// flight over their own ring of slots, each load landing on its slot's mbarrier; a thread waits
// for its oldest load before reusing the slot.  A load is box_rows rows x 128 B (2-D, 128-byte
// swizzle, as the contraction kernels' operand stages) or, with chunks > 1, a 3-D box of
// `chunks` consecutive 128-byte column blocks.  CTA c reads its own rows (`same` = 0) or every
// CTA reads the same rows (`same` = 1: a weight tile all CTAs share).  The data is not used.
constexpr int kTmaProbeSmemBytes = 196608;
constexpr int kTmaProbeMaxSlots = 16;

// MODE 0: the kernels' bounded wait (try_wait with timer checks); 1: a test_wait spin bounded
// by a count (never suspends).
template <int MODE>
__global__ void __launch_bounds__(128, 1)
    tma_rate_probe_kernel(const __grid_constant__ CUtensorMap tm, int box_rows, int chunks, int depth, int iters,
                          int row_blocks, int col_blocks, int same, int lanes_per_warp, unsigned long long* cycles,
                          unsigned long long* nanos, uint32_t* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kTmaProbeSmemBytes);
  volatile uint32_t* abort_flag = reinterpret_cast<uint32_t*>(full + kTmaProbeMaxSlots);
  // producers: lanes 0..lanes-1 of every warp (lanes = 1: lane 0 of each warp)
  const int lanes = lanes_per_warp;
  const int warps = (blockDim.x >> 5) * lanes;
  const int warp = (threadIdx.x >> 5) * lanes + static_cast<int>(threadIdx.x & 31);
  const uint32_t bytes = static_cast<uint32_t>(box_rows) * 128u * static_cast<uint32_t>(chunks);
  if (threadIdx.x == 0) {
    for (int i = 0; i < kTmaProbeMaxSlots; ++i) mbar_init(&full[i], 1);
    *abort_flag = 0u;
    fence_barrier_init();
    tma_prefetch_desc(&tm);
  }
  __syncthreads();
  if (static_cast<int>(threadIdx.x & 31) >= lanes) return;
  uint64_t* my_full = full + warp * depth;
  uint8_t* my_slots = smem + static_cast<size_t>(warp) * depth * bytes;
  const int base_rb = same ? 0 : static_cast<int>(blockIdx.x) * row_blocks;
  const int per_warp = iters / warps;
  bool ok = true;
  const unsigned long long g0 = globaltimer_ns();
  const long long c0 = clock64();
  for (int i = 0; i < per_warp + depth && ok; ++i) {
    if (i >= depth) {  // the load issued `depth` steps ago must land before its slot is reused
      const int j = i - depth;
      const uint32_t par = static_cast<uint32_t>((j / depth) & 1);
      if constexpr (MODE == 1) ok = spin_wait(&my_full[j % depth], par);
      else ok = mbar_wait(&my_full[j % depth], par, abort_flag, err);
    }
    if (i < per_warp) {
      const int slot = i % depth;
      const int g = i * warps + warp;  // load index across the CTA's producers
      const int cb = (g % (col_blocks / chunks)) * chunks;
      const int y = (base_rb + (g / (col_blocks / chunks)) % row_blocks) * box_rows;
      mbar_arrive_expect_tx(&my_full[slot], bytes);
      if (chunks == 1) tma_load_2d(&tm, &my_full[slot], my_slots + slot * bytes, cb * 128, y);
      else tma_load_3d(&tm, &my_full[slot], my_slots + slot * bytes, 0, y, cb);
    }
  }
  const long long c1 = clock64();
  const unsigned long long g1 = globaltimer_ns();
  if (!ok) {  // let the loads in flight land before the CTA exits
    volatile uint32_t no_abort = 0;
    for (int j = per_warp > depth ? per_warp - depth : 0; j < per_warp; ++j)
      mbar_wait(&my_full[j % depth], static_cast<uint32_t>((j / depth) & 1), &no_abort, err);
  }
  if (threadIdx.x == 0) {
    cycles[blockIdx.x] = ok ? static_cast<unsigned long long>(c1 - c0) : 0ull;
    nanos[blockIdx.x] = ok ? g1 - g0 : 0ull;
  }
}

// The same for im2col loads (the convolutions' A operand): an NHWC int8 tensor of 128
// channels, 3x3 filter, padding 1, stride 1; load g brings the 128 output pixels from
// (g * 128) mod (N*H*W) on, filter tap g mod 9, 128 channels: 16 KB.
__global__ void __launch_bounds__(128, 1)
    im2col_rate_probe_kernel(const __grid_constant__ CUtensorMap tm, int n, int h, int w, int depth, int iters,
                             unsigned long long* cycles, unsigned long long* nanos, uint32_t* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kTmaProbeSmemBytes);
  volatile uint32_t* abort_flag = reinterpret_cast<uint32_t*>(full + kTmaProbeMaxSlots);
  const int producers = blockDim.x >> 5;
  const int pr = threadIdx.x >> 5;
  constexpr uint32_t kBytes = 128u * 128u;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kTmaProbeMaxSlots; ++i) mbar_init(&full[i], 1);
    *abort_flag = 0u;
    fence_barrier_init();
    tma_prefetch_desc(&tm);
  }
  __syncthreads();
  if ((threadIdx.x & 31) != 0) return;
  uint64_t* my_full = full + pr * depth;
  uint8_t* my_slots = smem + static_cast<size_t>(pr) * depth * kBytes;
  const int pixels = n * h * w;
  const int per = iters / producers;
  bool ok = true;
  const unsigned long long g0 = globaltimer_ns();
  const long long c0 = clock64();
  for (int i = 0; i < per + depth && ok; ++i) {
    if (i >= depth) {
      const int j = i - depth;
      ok = mbar_wait(&my_full[j % depth], static_cast<uint32_t>((j / depth) & 1), abort_flag, err);
    }
    if (i < per) {
      const int slot = i % depth;
      const int g = (static_cast<int>(blockIdx.x) * per + i) * producers + pr;
      const int m0 = static_cast<int>((static_cast<long long>(g) * 128) % pixels);
      const int cn = m0 / (h * w);
      const int rem = m0 - cn * h * w;
      const int oy = rem / w, ox = rem - oy * w;
      const int tap = g % 9;
      mbar_arrive_expect_tx(&my_full[slot], kBytes);
      tma_load_im2col_4d(&tm, &my_full[slot], my_slots + slot * kBytes, 0, ox - 1, oy - 1, cn,
                         static_cast<uint16_t>(tap % 3), static_cast<uint16_t>(tap / 3));
    }
  }
  const long long c1 = clock64();
  const unsigned long long g1 = globaltimer_ns();
  if (!ok) {
    volatile uint32_t no_abort = 0;
    for (int j = per > depth ? per - depth : 0; j < per; ++j)
      mbar_wait(&my_full[j % depth], static_cast<uint32_t>((j / depth) & 1), &no_abort, err);
  }
  if (threadIdx.x == 0) {
    cycles[blockIdx.x] = ok ? static_cast<unsigned long long>(c1 - c0) : 0ull;
    nanos[blockIdx.x] = ok ? g1 - g0 : 0ull;
  }
}

}  // namespace
}  // namespace lsc

using namespace lsc;

extern "C" lsc_status lsc_probe_im2col_rate(const void* src, int64_t n, int64_t h, int64_t w, int32_t depth,
                                            int32_t producers, int32_t iters, int32_t ctas, double* bytes_per_clock,
                                            double* gbytes_per_s) {
  if (!src || (reinterpret_cast<uintptr_t>(src) & 127) || n < 1 || h < 3 || w < 3 || n * h * w > (1 << 26) ||
      depth < 1 || producers < 1 || producers > 4 || depth * producers > kTmaProbeMaxSlots ||
      16384LL * depth * producers > kTmaProbeSmemBytes || iters < producers || iters > (1 << 20) || ctas < 1 ||
      !bytes_per_clock || !gbytes_per_s)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "probe_im2col_rate: bad arguments");
  DeviceState* ds = current_device_state();
  if (!ds) return LSC_ERROR_DEVICE_ERROR;
  if (ds->cc_major != 10) return set_error(LSC_ERROR_BACKEND_NOT_AVAILABLE, "probe_im2col_rate: needs sm_100");
  const int units = ctas < ds->sm_count ? ctas : ds->sm_count;
  const uint64_t dims[4] = {128, static_cast<uint64_t>(w), static_cast<uint64_t>(h), static_cast<uint64_t>(n)};
  const uint64_t strides[3] = {128, static_cast<uint64_t>(w * 128), static_cast<uint64_t>(h * w * 128)};
  const int lower[2] = {-1, -1};
  const int upper[2] = {-1, -1};
  const uint32_t estr[4] = {1, 1, 1, 1};
  CUtensorMap tm;
  lsc_status st = encode_tmap_im2col(&tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, src, dims, strides, lower, upper, 128, 128,
                                     estr, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st) return st;
  const int smem = kTmaProbeSmemBytes + 1024 + 256;
  LSC_CUDA_TRY(cudaFuncSetAttribute(im2col_rate_probe_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  unsigned long long* buf = nullptr;
  LSC_CUDA_TRY(cudaMalloc(&buf, 2 * sizeof(unsigned long long) * units));
  im2col_rate_probe_kernel<<<units, 32 * producers, smem>>>(tm, static_cast<int>(n), static_cast<int>(h),
                                                             static_cast<int>(w), depth, iters, buf, buf + units,
                                                             ds->err_word);
  cudaError_t e = cudaGetLastError();
  std::vector<unsigned long long> hv(2 * units);
  if (e == cudaSuccess) e = cudaMemcpy(hv.data(), buf, hv.size() * sizeof(hv[0]), cudaMemcpyDeviceToHost);
  cudaFree(buf);
  if (e != cudaSuccess) return cuda_error(e, "probe_im2col_rate");
  std::vector<unsigned long long> c(hv.begin(), hv.begin() + units), t(hv.begin() + units, hv.end());
  if (std::find(c.begin(), c.end(), 0ull) != c.end())
    return set_error(LSC_ERROR_TIMEOUT, "probe_im2col_rate: a load wait ran out");
  std::sort(c.begin(), c.end());
  std::sort(t.begin(), t.end());
  const double moved = static_cast<double>(iters / producers * producers) * 16384.0;
  *bytes_per_clock = moved / static_cast<double>(c[units / 2]);
  *gbytes_per_s = moved * units / static_cast<double>(t[units / 2]);
  return LSC_SUCCESS;
}

extern "C" lsc_status lsc_probe_tma_rate(const void* src, uint64_t bytes, int64_t row_pitch, int32_t box_rows,
                                         int32_t chunks, int32_t depth, int32_t producers, int32_t same, int32_t iters,
                                         int32_t ctas, int32_t mode, double* bytes_per_clock, double* gbytes_per_s) {
  // mode 0 / 1: producers are lane 0 of `producers` warps; mode 2: lanes 0..producers-1 of one warp
  if (mode < 0 || mode > 2) return set_error(LSC_ERROR_INVALID_ARGUMENT, "probe_tma_rate: mode 0..2");
  const int warps = producers;
  if ((chunks != 1 && chunks != 2 && chunks != 4) || row_pitch < 128 * chunks)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "probe_tma_rate: chunks 1, 2 or 4 within the row");
  if (!src || (reinterpret_cast<uintptr_t>(src) & 127) || row_pitch < 128 || row_pitch % 128 ||
      (box_rows != 64 && box_rows != 128 && box_rows != 256) || depth < 1 || warps < 1 || warps > 4 ||
      warps * depth > kTmaProbeMaxSlots ||
      static_cast<int64_t>(box_rows) * 128 * chunks * depth * warps > kTmaProbeSmemBytes ||
      static_cast<int64_t>(box_rows) * 128 * chunks > 65536 || iters < warps || iters > (1 << 20) || ctas < 1 ||
      !bytes_per_clock || !gbytes_per_s)
    return set_error(LSC_ERROR_INVALID_ARGUMENT,
                     "probe_tma_rate: 128-byte aligned source, pitch a multiple of 128, box rows 64/128/256, "
                     "1..4 producer warps, slots within 192 KB, at most 64 KB per load, iters <= 2^20");
  DeviceState* ds = current_device_state();
  if (!ds) return LSC_ERROR_DEVICE_ERROR;
  if (ds->cc_major != 10) return set_error(LSC_ERROR_BACKEND_NOT_AVAILABLE, "probe_tma_rate: needs sm_100");
  const int units = ctas < ds->sm_count ? ctas : ds->sm_count;
  const int64_t rows = static_cast<int64_t>(bytes / static_cast<uint64_t>(row_pitch));
  const int col_blocks = static_cast<int>(row_pitch / 128);
  const int64_t row_blocks_total = rows / box_rows;
  const int row_blocks = static_cast<int>(same ? row_blocks_total : row_blocks_total / units);
  if (row_blocks < 1 || rows > INT32_MAX)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "probe_tma_rate: buffer too small (or too large) for the CTAs");
  CUtensorMap tm;
  lsc_status st;
  if (chunks == 1) {
    st = encode_tmap_2d(&tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, src, static_cast<uint64_t>(row_pitch),
                        static_cast<uint64_t>(rows), static_cast<uint64_t>(row_pitch), 128,
                        static_cast<uint32_t>(box_rows), CU_TENSOR_MAP_SWIZZLE_128B);
  } else {
    const uint64_t dims[3] = {128, static_cast<uint64_t>(rows), static_cast<uint64_t>(col_blocks)};
    const uint64_t strides[2] = {static_cast<uint64_t>(row_pitch), 128};
    const uint32_t box[3] = {128, static_cast<uint32_t>(box_rows), static_cast<uint32_t>(chunks)};
    const uint32_t estr[3] = {1, 1, 1};
    st = encode_tmap_3d(&tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, src, dims, strides, box, estr, CU_TENSOR_MAP_SWIZZLE_128B);
  }
  if (st) return st;
  const int smem = kTmaProbeSmemBytes + 1024 + 256;
  auto kernel = mode == 1 ? tma_rate_probe_kernel<1> : tma_rate_probe_kernel<0>;
  const int lanes = mode == 2 ? producers : 1;
  const int threads = mode == 2 ? 32 : 32 * producers;
  LSC_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  unsigned long long* buf = nullptr;
  LSC_CUDA_TRY(cudaMalloc(&buf, 2 * sizeof(unsigned long long) * units));
  kernel<<<units, threads, smem>>>(tm, box_rows, chunks, depth, iters, row_blocks, col_blocks, same, lanes, buf,
                                   buf + units, ds->err_word);
  cudaError_t e = cudaGetLastError();
  std::vector<unsigned long long> h(2 * units);
  if (e == cudaSuccess) e = cudaMemcpy(h.data(), buf, h.size() * sizeof(h[0]), cudaMemcpyDeviceToHost);
  cudaFree(buf);
  if (e != cudaSuccess) return cuda_error(e, "probe_tma_rate");
  std::vector<unsigned long long> c(h.begin(), h.begin() + units), t(h.begin() + units, h.end());
  if (std::find(c.begin(), c.end(), 0ull) != c.end())
    return set_error(LSC_ERROR_TIMEOUT, "probe_tma_rate: a load wait ran out");
  std::sort(c.begin(), c.end());
  std::sort(t.begin(), t.end());
  const double moved = static_cast<double>(iters / warps * warps) * box_rows * 128.0 * chunks;
  *bytes_per_clock = moved / static_cast<double>(c[units / 2]);
  *gbytes_per_s = moved * units / static_cast<double>(t[units / 2]);
  return LSC_SUCCESS;
}

extern "C" lsc_status lsc_probe_tensor_rate(int32_t kind, int32_t n, int32_t cta_pair, int32_t iters, int32_t ctas,
                                            int32_t mode, int32_t commit_every, int32_t wait_lag,
                                            double* cycles_per_mma, double* ns_per_mma) {
  if ((kind != 0 && kind != 1) || iters < 1 || iters > (1 << 22) || ctas < 1 || !cycles_per_mma || !ns_per_mma ||
      commit_every < 0 || wait_lag < 0 || wait_lag > 7)
    return set_error(LSC_ERROR_INVALID_ARGUMENT,
                     "probe_tensor_rate: kind 0|1, 1 <= iters <= 2^22, ctas >= 1, commit_every >= 0, wait_lag 0..7");
  DeviceState* ds = current_device_state();
  if (!ds) return LSC_ERROR_DEVICE_ERROR;
  if (ds->cc_major != 10) return set_error(LSC_ERROR_BACKEND_NOT_AVAILABLE, "probe_tensor_rate: needs sm_100");
  const int units = cta_pair ? std::min(ctas, ds->sm_count / 2) : std::min(ctas, ds->sm_count);
  unsigned long long* buf = nullptr;
  LSC_CUDA_TRY(cudaMalloc(&buf, 2 * sizeof(unsigned long long) * units));
  lsc_status st;
  const int ce = commit_every, lag = wait_lag;
  unsigned long long* cyc = buf;
  unsigned long long* nan = buf + units;
  uint32_t* ew = ds->err_word;
  if (kind == 0) st = cta_pair ? run_probe_mode<0, true>(mode, n, iters, ce, lag, units, cyc, nan, ew)
                               : run_probe_mode<0, false>(mode, n, iters, ce, lag, units, cyc, nan, ew);
  else st = cta_pair ? run_probe_mode<1, true>(mode, n, iters, ce, lag, units, cyc, nan, ew)
                     : run_probe_mode<1, false>(mode, n, iters, ce, lag, units, cyc, nan, ew);
  std::vector<unsigned long long> h(2 * units);
  if (st == LSC_SUCCESS) {
    cudaError_t e = cudaMemcpy(h.data(), buf, h.size() * sizeof(h[0]), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) st = cuda_error(e, "probe_tensor_rate: result copy");
  }
  cudaFree(buf);
  if (st) return st;
  std::vector<unsigned long long> c(h.begin(), h.begin() + units), t(h.begin() + units, h.end());
  if (std::find(c.begin(), c.end(), 0ull) != c.end())
    return set_error(LSC_ERROR_TIMEOUT, "probe_tensor_rate: a completion wait ran out");
  std::sort(c.begin(), c.end());
  std::sort(t.begin(), t.end());
  const int issued = mode >= 2 ? iters / 4 * 4 : iters;
  *cycles_per_mma = static_cast<double>(c[units / 2]) / issued;
  *ns_per_mma = static_cast<double>(t[units / 2]) / issued;
  return LSC_SUCCESS;
}
