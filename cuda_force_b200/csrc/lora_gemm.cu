// LoRA linear on the 5th-generation tensor cores (tcgen05 + TMEM + TMA), sm_100a.
//
//   y[m, n] = sum_k x[m,k] W[k,n] + scale * sum_j (sum_k x[m,k] A[k,j]) B[j,n]
//
// Semantics follow the reference's lora_linear (python/cudaforge/ops.py:178-185,
// cpp/src/bindings.cpp:255-258, CUDA launcher cuda/src/lora_linear.cu:237-277);
// the W8 variant computes lora_linear(x, dequantize_int8(codes, scales)^T, ...)
// with the reference's dequantisation (bindings.cpp:320-329) applied in shared
// memory: q * s in fp32 exactly as the dequantiser does, then rounded to the
// activation dtype for the MMA.
//
// Two launches per call, the second allowed to start while the first runs
// (programmatic dependent launch; it waits for the first only before reading P):
//   1. down-projection  P = scale * x A  -> workspace [M, r] (bf16/f16), split-K
//      over a thread-block cluster (down_proj_kernel);
//   2. main product     y = x W^T + P B  with the adapter folded into the MMA as
//      r/16 extra K-steps (P and the B slice as operands), so the rank-r update
//      costs no epilogue arithmetic:
//        lora_gemm_kernel   bf16/f16 W, 128 x BN tiles of y, persistent;
//        w8_wide_kernel     int8 W, M > 128: swap-AB 128-feature x 512-token
//                           tiles, codes converted to bf16/f16 in shared memory
//                           by eight converter warps, persistent; also the
//                           fused all-gather (TMA-store epilogue to every
//                           destination);
//        w8_decode_kernel   int8 W, M <= 128: one 128-feature tile per CTA with
//                           K split across a cluster and a DSMEM reduction.
// Roles: one TMA producer thread, one MMA-issuing thread that also owns TMEM,
// four TMEM-reading epilogue warps (thread = accumulator lane), and for int8
// weights eight converter warps. Every mbarrier wait is bounded (2 s of global
// time); on expiry the kernel records CF_ERR_DEVICE_TIMEOUT in the device error
// word and unwinds.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <atomic>
#include <cstring>
#include <mutex>

#include "cf_common.cuh"
#include "ptx.cuh"
#include "quant_math.cuh"

namespace cfb {
namespace {

constexpr int kBM = 128;        // tile rows (MMA M)
constexpr int kBK = 64;         // k-block: 64 x 16-bit = one 128-byte swizzle row
constexpr int kUmmaK = 16;      // K per tcgen05.mma (kind::f16)
constexpr int kEpiWarp0 = 4;    // first epilogue warp (warp % 4 = TMEM lane quarter)
constexpr int kConvWarp0 = 8;   // first converter warp (W8 only)
constexpr int kConvThreads = 256;

enum BSource : int { kBKMajor = 0, kBMNMajor = 1 };

template <int BN>
struct GemmCfg {
  static constexpr int kABytes = kBM * kBK * 2;                // 16 KB
  static constexpr int kBBytes = (BN < 64 ? 64 : BN) * kBK * 2;  // >= 8 KB so extras fit
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = BN >= 128 ? 4 : 8;
  static constexpr int kThreads = 256;
  static constexpr int kTmemCols = (2 * BN) <= 32 ? 32 : (2 * BN) <= 64 ? 64
                                   : (2 * BN) <= 128 ? 128 : (2 * BN) <= 256 ? 256 : 512;
  static constexpr size_t kSmemBytes = 1024 /*alignment slack*/ +
                                       static_cast<size_t>(kStages) * kStageBytes + 256;
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "MMA N");
};

struct GemmParams {
  int M, N, K;
  int num_kb;          // ceil(K / 64)
  int extra_ksteps;    // adapter K-steps (rank / 16); 0 = none
  int rank;            // adapter rank (16, 32 or 64)
  int b_src;           // BSource of the main B operand
  int extra_b_mn;      // adapter B operand stored MN-major ([rank, N])
  int is_bf16;
  float out_scale;     // multiplier applied in the epilogue
  void *out;           // [M, ldo] row-major, 16-bit
  int ldo;
  int n_tiles_n;
  int n_tiles;
  unsigned *err;
};

__device__ __forceinline__ uint32_t swizzle_for_row_bytes(int row_bytes) {
  return row_bytes >= 128 ? ptx::kSwizzle128B : row_bytes == 64 ? ptx::kSwizzle64B
                                                                 : ptx::kSwizzle32B;
}

// Shared-memory descriptor of a K-major operand whose rows are `row_bytes`
// (32/64/128) long and swizzled at that width; 8-row core groups are
// 8 * row_bytes apart. k-step `ks` (16 elements = 32 bytes) advances the start
// address inside the swizzle atom.
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t base, int row_bytes, int ks) {
  return ptx::make_smem_desc(base + ks * 32, 16, 8 * row_bytes, swizzle_for_row_bytes(row_bytes));
}

// Descriptor of an MN-major operand stored as chunks of `chunk_elems` MN
// elements (chunk_elems * 2 = row bytes, swizzled at that width) x k rows;
// chunks are `chunk_stride` bytes apart. k-step `ks` = 16 rows further.
__device__ __forceinline__ uint64_t mnmajor_desc(uint32_t base, int row_bytes, int chunk_stride,
                                                 int ks) {
  return ptx::make_smem_desc(base + ks * 16 * row_bytes, chunk_stride, 8 * row_bytes,
                             swizzle_for_row_bytes(row_bytes));
}

__device__ __forceinline__ void record_timeout(unsigned *err, int *abort_flag) {
  atomicOr(err, kDevErrTimeout);
  *reinterpret_cast<volatile int *>(abort_flag) = 1;
}

__device__ __forceinline__ bool aborted(const int *abort_flag) {
  return *reinterpret_cast<const volatile int *>(abort_flag) != 0;
}

// Tile t of a grid of `rows` x `cols` tiles, walked in bands of `band` rows
// with the row index fastest inside a band: the CTAs of one wave then share
// a few column blocks (each read from DRAM about once per band) while the
// band's row blocks stay resident in L2.
__device__ __forceinline__ void band_order(int t, int rows, int cols, int band, int &row,
                                           int &col) {
  const int per_band = band * cols;
  const int b = t / per_band;
  const int in_band = min(band, rows - b * band);
  const int i = t - b * per_band;
  row = b * band + i % in_band;
  col = i / in_band;
}

template <int BN, bool kBf16>
__global__ void __launch_bounds__(GemmCfg<BN>::kThreads, 1)
    lora_gemm_kernel(const __grid_constant__ CUtensorMap tm_a,
                     const __grid_constant__ CUtensorMap tm_b,
                     const __grid_constant__ CUtensorMap tm_pa,
                     const __grid_constant__ CUtensorMap tm_pb, const GemmParams p) {
  using C = GemmCfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::kStages * C::kStageBytes);
  uint64_t *full = bars;                       // [kStages] TMA -> consumers
  uint64_t *empty = bars + C::kStages;         // [kStages] MMA -> producer
  uint64_t *tmem_full = bars + 2 * C::kStages; // [2] MMA -> epilogue
  uint64_t *tmem_empty = tmem_full + 2;        // [2] epilogue -> MMA
  uint64_t *drain = tmem_empty + 2;             // [1] MMA retirement on abort
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
  int *abort_flag = reinterpret_cast<int *>(tmem_slot + 1);

  const int warp = threadIdx.x / kWarp;
  const int lane = threadIdx.x % kWarp;
  const int num_iters = p.num_kb + (p.extra_ksteps > 0 ? 1 : 0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      ptx::mbar_init(&full[s], 1);
      ptx::mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      ptx::mbar_init(&tmem_full[a], 1);
      ptx::mbar_init(&tmem_empty[a], 4);
    }
    ptx::mbar_init(drain, 1);
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    ptx::prefetch_tensor_map(&tm_a);
    ptx::prefetch_tensor_map(&tm_b);
    if (p.extra_ksteps > 0) {
      ptx::prefetch_tensor_map(&tm_pa);
      ptx::prefetch_tensor_map(&tm_pb);
    }
  }
  if (warp == 1) {
    ptx::tmem_alloc(tmem_slot, C::kTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t outstanding = 0, issue_parity = 0;
      bool dep_ready = false;
      const int extra_a_bytes = kBM * p.rank * 2;
      const int extra_b_bytes = BN * p.rank * 2;
      for (int tile = blockIdx.x; tile < p.n_tiles && !aborted(abort_flag); tile += gridDim.x) {
        const int m0 = (tile / p.n_tiles_n) * kBM;
        const int n0 = (tile % p.n_tiles_n) * BN;
        for (int it = 0; it < num_iters; ++it) {
          if (!ptx::mbar_wait(&empty[stage], phase ^ 1)) {
            record_timeout(p.err, abort_flag);
            break;
          }
          uint8_t *sa = smem + stage * C::kStageBytes;
          uint8_t *sb = sa + C::kABytes;
          if (it < p.num_kb) {
            const int k0 = it * kBK;
            ptx::mbar_expect_tx(&full[stage], C::kABytes + BN * kBK * 2);
            ptx::tma_load_2d(sa, &tm_a, &full[stage], k0, m0);
            if (p.b_src == kBMNMajor) {
              // chunks of min(BN, 64) columns x 64 k-rows, one swizzle row each
              constexpr int kChunkCols = BN < 64 ? BN : 64;
              for (int c = 0; c < BN / kChunkCols; ++c) {
                ptx::tma_load_2d(sb + c * (kBK * kChunkCols * 2), &tm_b, &full[stage],
                                 n0 + c * kChunkCols, k0);
              }
            } else {
              ptx::tma_load_2d(sb, &tm_b, &full[stage], k0, n0);
            }
          } else {
            if (!dep_ready) {  // P comes from the down-projection launched just before
              ptx::grid_dep_wait();
              dep_ready = true;
            }
            ptx::mbar_expect_tx(&full[stage], extra_a_bytes + extra_b_bytes);
            ptx::tma_load_2d(sa, &tm_pa, &full[stage], 0, m0);
            if (p.extra_b_mn) {
              for (int c = 0; c < BN / 64; ++c) {
                ptx::tma_load_2d(sb + c * (p.rank * 128), &tm_pb, &full[stage], n0 + c * 64, 0);
              }
            } else {
              ptx::tma_load_2d(sb, &tm_pb, &full[stage], 0, n0);
            }
          }
          outstanding |= 1u << stage;
          issue_parity = (issue_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (aborted(abort_flag)) {
        // Let loads already issued land before the CTA's shared memory goes away.
        for (int s = 0; s < C::kStages; ++s) {
          if (outstanding & (1u << s)) ptx::mbar_wait(&full[s], (issue_parity >> s) & 1u, 200000000ull);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const bool bf16 = kBf16;
      const uint32_t idesc_main = ptx::make_idesc_f16(bf16, kBM, BN, false, p.b_src == kBMNMajor);
      const uint32_t idesc_extra = ptx::make_idesc_f16(bf16, kBM, BN, false, p.extra_b_mn != 0);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      for (int tile = blockIdx.x; tile < p.n_tiles && !aborted(abort_flag);
           tile += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = static_cast<uint32_t>((local >> 1) & 1);
        if (!ptx::mbar_wait(&tmem_empty[acc], acc_phase ^ 1)) {
          record_timeout(p.err, abort_flag);
          break;
        }
        ptx::tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        bool ok = true;
        for (int it = 0; it < num_iters; ++it) {
          const bool main_kb = it < p.num_kb;
          if (!ptx::mbar_wait(&full[stage], phase)) {
            record_timeout(p.err, abort_flag);
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          const uint32_t sa = ptx::smem_addr(smem + stage * C::kStageBytes);
          const uint32_t sb = sa + C::kABytes;
          if (main_kb) {
            for (int ks = 0; ks < kBK / kUmmaK; ++ks) {
              const uint64_t adesc = kmajor_desc(sa, 128, ks);
              constexpr int kChunkCols = BN < 64 ? BN : 64;
              const uint64_t bdesc =
                  p.b_src == kBMNMajor ? mnmajor_desc(sb, kChunkCols * 2, kBK * kChunkCols * 2, ks)
                                       : kmajor_desc(sb, 128, ks);
              ptx::mma_f16(d_tmem, adesc, bdesc, idesc_main, (it > 0 || ks > 0) ? 1u : 0u);
            }
          } else {
            const int row_bytes = p.rank * 2;
            for (int ks = 0; ks < p.extra_ksteps; ++ks) {
              const uint64_t adesc = kmajor_desc(sa, row_bytes, ks);
              const uint64_t bdesc = p.extra_b_mn ? mnmajor_desc(sb, 128, p.rank * 128, ks)
                                                  : kmajor_desc(sb, row_bytes, ks);
              ptx::mma_f16(d_tmem, adesc, bdesc, idesc_extra, (it > 0 || ks > 0) ? 1u : 0u);
            }
          }
          ptx::mma_commit(&empty[stage]);
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        ptx::mma_commit(&tmem_full[acc]);
      }
      if (aborted(abort_flag)) {
        // Retire MMAs still in flight before TMEM is released.
        ptx::mma_commit(drain);
        ptx::mbar_wait(drain, 0, 200000000ull);
      }
    }
  } else if (warp >= kEpiWarp0 && warp < kEpiWarp0 + 4) {
    // ------------------------------------------------------------------ epilogue
    const int quarter = warp % 4;
    int local = 0;
    for (int tile = blockIdx.x; tile < p.n_tiles; tile += gridDim.x, ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = static_cast<uint32_t>((local >> 1) & 1);
      const bool ok = ptx::warp_wait(&tmem_full[acc], acc_phase);
      if (__any_sync(0xffffffffu, !ok)) {
        if (lane == 0) record_timeout(p.err, abort_flag);
        break;
      }
      ptx::tc_fence_after();
      const int m0 = (tile / p.n_tiles_n) * kBM;
      const int n0 = (tile % p.n_tiles_n) * BN;
      const int row = m0 + quarter * 32 + lane;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * BN;
      uint16_t *out_row = static_cast<uint16_t *>(p.out) + static_cast<int64_t>(row) * p.ldo;
      constexpr int kChunk = BN >= 32 ? 32 : 16;
#pragma unroll 1
      for (int c = 0; c < BN / kChunk; ++c) {
        uint32_t v[32];
        if constexpr (kChunk == 32) {
          ptx::tmem_ld_32x32b_x32(t_row + c * 32, v);
        } else {
          ptx::tmem_ld_32x32b_x16(t_row + c * 16, v);
        }
        ptx::tmem_ld_wait();
        uint32_t packed[kChunk / 2];
#pragma unroll
        for (int e = 0; e < kChunk / 2; ++e) {
          const float lo = __uint_as_float(v[2 * e]) * p.out_scale;
          const float hi = __uint_as_float(v[2 * e + 1]) * p.out_scale;
          packed[e] = kBf16 ? ptx::pack_bf16x2(lo, hi) : ptx::pack_f16x2(lo, hi);
        }
        if (row < p.M) {
          const int col0 = n0 + c * kChunk;
#pragma unroll
          for (int q = 0; q < kChunk / 8; ++q) {
            if (col0 + q * 8 < p.N) {
              *reinterpret_cast<uint4 *>(out_row + col0 + q * 8) =
                  make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
            }
          }
        }
      }
      ptx::tc_fence_before();
      ptx::warp_arrive(&tmem_empty[acc]);
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem_base, C::kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// Down-projection P = scale * x A with split-K across a thread-block cluster.
//
// One cluster per 128-row tile of x; its S CTAs take consecutive slices of K,
// accumulate 128 x R partial sums in TMEM (tcgen05.mma, N = R), park them in
// shared memory, and after a cluster barrier each CTA reduces 128/S rows across
// the S partials through distributed shared memory, scales, rounds and stores
// its rows of P. No global scratch, deterministic summation order, and small M
// (decode) still spreads the x and A stream over S SMs.
//   warp 0: TMA producer; warp 1: TMEM owner + MMA issuer; warps 2-5: epilogue.
// ---------------------------------------------------------------------------
template <int R>
struct DownCfg {
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = R * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = 8;
  static constexpr int kPartialBytes = kBM * R * 4;
  static constexpr int kThreads = 192;
  static constexpr int kTmemCols = R < 32 ? 32 : R;
  static constexpr size_t kSmemBytes =
      1024 + static_cast<size_t>(kStages) * kStageBytes + kPartialBytes + 256;
};

struct DownParams {
  int M;
  int num_kb;
  int kb_per_split;
  int splits;
  int a_mn_major;  // A stored [K, r] (r contiguous)
  float scale;
  void *out;  // P [M, R] 16-bit
  unsigned *err;
};

template <int R, bool kBf16>
__global__ void __launch_bounds__(DownCfg<R>::kThreads, 1)
    down_proj_kernel(const __grid_constant__ CUtensorMap tm_x,
                     const __grid_constant__ CUtensorMap tm_a, const DownParams p) {
  using C = DownCfg<R>;
  // The linear kernel that consumes P may start now: it streams its main loop
  // and waits for this grid only before its first read of P.
  ptx::grid_dep_launch_dependents();
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  float *partial = reinterpret_cast<float *>(smem + C::kStages * C::kStageBytes);
  uint64_t *bars = reinterpret_cast<uint64_t *>(partial + kBM * R);
  uint64_t *full = bars;
  uint64_t *empty = bars + C::kStages;
  uint64_t *acc_full = bars + 2 * C::kStages;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_full + 1);
  int *abort_flag = reinterpret_cast<int *>(tmem_slot + 1);

  const int warp = threadIdx.x / kWarp;
  const int lane = threadIdx.x % kWarp;
  const int rank = static_cast<int>(ptx::cluster_ctarank());
  const int m0 = (blockIdx.x / p.splits) * kBM;
  const int kb0 = rank * p.kb_per_split;
  const int nkb = max(0, min(p.num_kb, kb0 + p.kb_per_split) - kb0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      ptx::mbar_init(&full[s], 1);
      ptx::mbar_init(&empty[s], 1);
    }
    ptx::mbar_init(acc_full, 1);
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == 1) {
    ptx::tmem_alloc(tmem_slot, C::kTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t outstanding = 0, issue_parity = 0;
      for (int i = 0; i < nkb; ++i) {
        if (!ptx::mbar_wait(&empty[stage], phase ^ 1)) {
          record_timeout(p.err, abort_flag);
          break;
        }
        uint8_t *sa = smem + stage * C::kStageBytes;
        const int k0 = (kb0 + i) * kBK;
        ptx::mbar_expect_tx(&full[stage], C::kStageBytes);
        ptx::tma_load_2d(sa, &tm_x, &full[stage], k0, m0);
        if (p.a_mn_major) {
          ptx::tma_load_2d(sa + C::kABytes, &tm_a, &full[stage], 0, k0);
        } else {
          ptx::tma_load_2d(sa + C::kABytes, &tm_a, &full[stage], k0, 0);
        }
        outstanding |= 1u << stage;
        issue_parity = (issue_parity & ~(1u << stage)) | (phase << stage);
        if (++stage == C::kStages) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (aborted(abort_flag)) {
        for (int s = 0; s < C::kStages; ++s) {
          if (outstanding & (1u << s)) ptx::mbar_wait(&full[s], (issue_parity >> s) & 1u, 200000000ull);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && nkb > 0) {
      const uint32_t idesc = ptx::make_idesc_f16(kBf16, kBM, R, false, p.a_mn_major != 0);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int i = 0; i < nkb; ++i) {
        if (!ptx::mbar_wait(&full[stage], phase)) {
          record_timeout(p.err, abort_flag);
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        const uint32_t sa = ptx::smem_addr(smem + stage * C::kStageBytes);
        const uint32_t sb = sa + C::kABytes;
        for (int ks = 0; ks < kBK / kUmmaK; ++ks) {
          const uint64_t adesc = kmajor_desc(sa, 128, ks);
          const uint64_t bdesc = p.a_mn_major ? mnmajor_desc(sb, R * 2, C::kBBytes, ks)
                                              : kmajor_desc(sb, 128, ks);
          ptx::mma_f16(tmem_base, adesc, bdesc, idesc, (i > 0 || ks > 0) ? 1u : 0u);
        }
        ptx::mma_commit(&empty[stage]);
        if (++stage == C::kStages) {
          stage = 0;
          phase ^= 1;
        }
      }
      // Also retires everything issued when aborting, before TMEM is freed.
      ptx::mma_commit(acc_full);
      if (!ok) ptx::mbar_wait(acc_full, 0, 200000000ull);
    }
  } else {
    // epilogue warps 2..5 cover the four TMEM lane quarters
    const int quarter = warp % 4;
    const int row = quarter * 32 + lane;
    float *prow = partial + row * R;
    bool have = nkb > 0;
    if (have) {
      const bool ok = ptx::mbar_wait(acc_full, 0);
      if (__any_sync(0xffffffffu, !ok)) {
        if (lane == 0) record_timeout(p.err, abort_flag);
        have = false;
      }
    }
    if (have) {
      ptx::tc_fence_after();
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
#pragma unroll
      for (int c = 0; c < (R + 31) / 32; ++c) {
        uint32_t v[32];
        if constexpr (R >= 32) {
          ptx::tmem_ld_32x32b_x32(t_row + c * 32, v);
        } else {
          ptx::tmem_ld_32x32b_x16(t_row, v);
        }
        ptx::tmem_ld_wait();
        constexpr int kCols = R >= 32 ? 32 : R;
#pragma unroll
        for (int e = 0; e < kCols; e += 4) {
          *reinterpret_cast<float4 *>(prow + c * 32 + e) =
              make_float4(__uint_as_float(v[e]), __uint_as_float(v[e + 1]),
                          __uint_as_float(v[e + 2]), __uint_as_float(v[e + 3]));
        }
      }
    } else {
#pragma unroll
      for (int e = 0; e < R; e += 4) *reinterpret_cast<float4 *>(prow + e) = make_float4(0, 0, 0, 0);
    }
  }

  // Partials of every CTA are in shared memory; reduce across the cluster.
  ptx::tc_fence_before();
  ptx::cluster_sync();
  {
    const int rows_per = kBM / p.splits;
    const int r_begin = rank * rows_per;
    const int items = rows_per * (R / 4);
    const uint32_t base = ptx::smem_addr(partial);
    for (int it = threadIdx.x; it < items; it += C::kThreads) {
      const int row = r_begin + it / (R / 4);
      const int c4 = (it % (R / 4)) * 4;
      const uint32_t off = static_cast<uint32_t>((row * R + c4) * 4);
      float4 acc = make_float4(0, 0, 0, 0);
      for (int peer = 0; peer < p.splits; ++peer) {
        const float4 v = ptx::ld_shared_cluster_f4(ptx::map_shared_rank(base + off, peer));
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
      }
      const int grow = m0 + row;
      if (grow < p.M) {
        const uint32_t lo = kBf16 ? ptx::pack_bf16x2(acc.x * p.scale, acc.y * p.scale)
                                  : ptx::pack_f16x2(acc.x * p.scale, acc.y * p.scale);
        const uint32_t hi = kBf16 ? ptx::pack_bf16x2(acc.z * p.scale, acc.w * p.scale)
                                  : ptx::pack_f16x2(acc.z * p.scale, acc.w * p.scale);
        *reinterpret_cast<uint2 *>(static_cast<uint16_t *>(p.out) + static_cast<int64_t>(grow) * R +
                                   c4) = make_uint2(lo, hi);
      }
    }
  }
  // No CTA may leave while a peer can still read its shared memory.
  ptx::cluster_sync();
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem_base, C::kTmemCols);
  }
}

constexpr int kMaxOuts = 8;

struct W8Params {
  int M;             // tokens
  int N;             // output features (rows of W)
  int num_kb;        // k-blocks of 32
  int extra_ksteps;  // rank / 16
  int rank;
  int extra_b_mn;    // B stored [rank, N] (N contiguous)
  const float *w_scales;
  int kb_per_row;    // scales per row (K / 64)
  int scale_tma;     // scales arrive by TMA with each stage (kb_per_row % 4 == 0)
  int ldo;           // row stride of every destination (elements)
  int out_col0;      // first column of this call's features in the destination
  int n_outs;        // destinations written by the epilogue
  int self_out;      // index of the destination on this GPU (stored first)
  void *outs[kMaxOuts];
  // Multicast address of the destination (all ranks' y bound to one NVLink
  // multicast object); when set, the epilogue writes every slab once with
  // multimem stores instead of one TMA store per destination.
  void *mc_out;
  // Folded RMSNorm (kNorm): each code is also multiplied by the norm weight of
  // its input feature, and each token's output by its row scale.
  const float *norm_w;      // [K] fp32
  const float *row_scale;   // [M]
  int n_tiles_w;
  int n_tiles;
  unsigned *err;
  // Row-group completion counters (wide kernel, copy-engine all-gather):
  // after a tile's stores have landed, done[row_block / rb_per_group] += 1.
  unsigned *done;
  int rb_per_group;
  int n_groups;
};

// ---------------------------------------------------------------------------
// W8 + LoRA for decode-sized token counts (M <= 128): one 128-feature tile
// per CTA, K split across a thread-block cluster.
//
// Decode is an HBM stream of int8 codes, so the kernel keeps the stream
// moving with three independent rings, each freed by its last reader:
//   raw   128 x 128 int8 code tiles (two k-blocks, 16 KB: 128-byte row
//         segments), loaded by TMA and released by the converter warps once
//         both k-blocks are converted;
//   x     BT x 64 activation tiles, loaded by a second TMA thread and
//         released by the MMA;
//   conv  128 x 64 bf16/f16 weight tiles written by the converters and
//         released by the MMA.
// Each CTA accumulates its K slice of the 128 x BT tile in TMEM (swap-AB: W
// tile = A operand, tokens = N). The cluster's rank-0 CTA then adds the
// rank-r adapter as rank/16 more K-steps: the code producer loads the tile's
// B^T slice into the next raw slot and the activation producer, once the
// down-projection grid has completed, loads P = (alpha/r) x A into the next
// activation slot. Every CTA parks its fp32 partial over its spent rings,
// and after a cluster barrier reduces a share of the rows across the cluster
// through distributed shared memory and writes them.
//   warp 0 code producer, warp 1 TMEM owner + MMA issuer, warp 2 activation
//   producer, warps 4-7 TMEM readers, warps 8-15 converters; all reduce.
// ---------------------------------------------------------------------------

// Ring waits in the decode kernel poll (no suspend hint): nearly every one of
// them blocks on memory, and polling resumes as soon as the phase flips.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

template <int BT>
struct DecCfg {
  // A raw stage holds kRawKb k-blocks: 128-byte row segments, so one TMA box
  // moves 16 KB in 128 row requests.
  static constexpr int kRawKb = 2;
  static constexpr int kRawBytes = kBM * kBK * kRawKb;  // 16 KB int8 codes
  static constexpr int kXBytes = BT * kBK * 2;          // activation tile
  static constexpr int kConvBytes = kBM * kBK * 2;      // 16 KB converted tile
  // BT = 32: three raw stages (six k-blocks, 48 KB per CTA, still far more
  // than the bandwidth-latency product needs at two CTAs per SM) and three
  // converted slots, so the converters run two k-blocks ahead of the MMA's
  // commit instead of one (3 % faster than 4 + 2 at x [32, 4096], W [11008, 4096]).
  static constexpr int kRawStages = BT <= 32 ? 3 : 2;
  static constexpr int kXStages = BT <= 64 ? 2 : 2;
  static constexpr int kConvSlots = BT <= 64 ? 3 : 2;
  // Each raw stage also carries the tile's scales: 128 rows x 4 k-blocks of
  // fp32 (a 16-byte TMA row; the stage's two k-blocks sit inside it), so no
  // converter waits on a global load of its scale.
  static constexpr int kScaleBytes = kBM * 4 * 4;  // 2 KB
  static constexpr int kRawOff = 0;
  static constexpr int kScaleOff = kRawOff + kRawStages * kRawBytes;
  static constexpr int kXOff = kScaleOff + kRawStages * kScaleBytes;
  static constexpr int kConvOff = kXOff + kXStages * kXBytes;
  static constexpr int kRingBytes = kConvOff + kConvSlots * kConvBytes;
  static constexpr int kPartialBytes = kBM * BT * 4;  // aliases the spent rings
  static_assert(kPartialBytes <= kRingBytes, "partial tile must fit in the rings");
  // Adapter operands: B^T slice (128 x rank <= 64) in a raw slot, P (BT x
  // rank) in an activation slot.
  static_assert(kBM * 64 * 2 <= kRawBytes && BT * 64 * 2 <= kXBytes, "adapter tiles");
  static_assert(kXOff % 1024 == 0 && kConvOff % 1024 == 0, "ring alignment");
  static constexpr int kThreads = 512;
  static constexpr int kMinBlocks = 2;  // two CTAs per SM: twice the loads in flight
  static constexpr int kTmemCols = BT < 32 ? 32 : BT;
  static constexpr size_t kSmemBytes = 1024 + static_cast<size_t>(kRingBytes) + 256;
};

struct DecParams {
  int M, N;
  int num_kb;        // k-blocks of 64
  int kb_per_split;
  int splits;        // cluster size
  int rank;          // adapter rank (16, 32 or 64)
  int b_mn;          // b stored [rank, N] (N contiguous: MN-major A operand)
  int scale_tma;     // scales arrive by TMA with the codes (num_kb % 4 == 0)
  const float *w_scales;
  uint16_t *out;     // y [M, N]
  unsigned *err;
};

template <int BT, bool kBf16>
__global__ void __launch_bounds__(DecCfg<BT>::kThreads, DecCfg<BT>::kMinBlocks)
    w8_decode_kernel(const __grid_constant__ CUtensorMap tm_x,
                     const __grid_constant__ CUtensorMap tm_codes,
                     const __grid_constant__ CUtensorMap tm_p,
                     const __grid_constant__ CUtensorMap tm_bt,
                     const __grid_constant__ CUtensorMap tm_scales, const DecParams p) {
  using C = DecCfg<BT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t *raw_ring = smem + C::kRawOff;
  const float *scale_ring = reinterpret_cast<const float *>(smem + C::kScaleOff);
  uint8_t *x_ring = smem + C::kXOff;
  uint8_t *conv = smem + C::kConvOff;
  float *partial = reinterpret_cast<float *>(smem);
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::kRingBytes);
  uint64_t *raw_full = bars;
  uint64_t *raw_empty = raw_full + C::kRawStages;
  uint64_t *x_full = raw_empty + C::kRawStages;
  uint64_t *x_empty = x_full + C::kXStages;
  uint64_t *conv_full = x_empty + C::kXStages;
  uint64_t *conv_empty = conv_full + C::kConvSlots;
  uint64_t *tmem_full = conv_empty + C::kConvSlots;
  uint64_t *drain = tmem_full + 1;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
  int *abort_flag = reinterpret_cast<int *>(tmem_slot + 1);
  constexpr int kConvWarps = kConvThreads / kWarp;

  const int warp = threadIdx.x / kWarp;
  const int lane = threadIdx.x % kWarp;
  const int rank = static_cast<int>(ptx::cluster_ctarank());
  const int tile = static_cast<int>(blockIdx.x) / p.splits;
  const int w0 = tile * kBM;
  const int kb0 = rank * p.kb_per_split;
  const int nkb = max(0, min(p.num_kb, kb0 + p.kb_per_split) - kb0);
  const bool adapter = rank == 0;  // this CTA adds the rank-r term
  const int n_raw_loads = (nkb + C::kRawKb - 1) / C::kRawKb;

  if (threadIdx.x == 0) {
    // Descriptor fetches overlap the setup instead of the first loads.
    ptx::prefetch_tensor_map(&tm_codes);
    ptx::prefetch_tensor_map(&tm_x);
    ptx::prefetch_tensor_map(&tm_p);
    ptx::prefetch_tensor_map(&tm_bt);
    if (p.scale_tma) ptx::prefetch_tensor_map(&tm_scales);
    for (int s = 0; s < C::kRawStages; ++s) {
      ptx::mbar_init(&raw_full[s], 1);
      ptx::mbar_init(&raw_empty[s], kConvWarps);
    }
    for (int s = 0; s < C::kXStages; ++s) {
      ptx::mbar_init(&x_full[s], 1);
      ptx::mbar_init(&x_empty[s], 1);
    }
    for (int c = 0; c < C::kConvSlots; ++c) {
      ptx::mbar_init(&conv_full[c], kConvWarps);
      ptx::mbar_init(&conv_empty[c], 1);
    }
    ptx::mbar_init(tmem_full, 1);
    ptx::mbar_init(drain, 1);
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == 1) {
    ptx::tmem_alloc(tmem_slot, C::kTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0 || warp == 2) {
    // ------------------------------------------------- producers (codes / x)
    if (lane == 0) {
      const bool codes = warp == 0;
      const int n_stages = codes ? C::kRawStages : C::kXStages;
      uint64_t *full = codes ? raw_full : x_full;
      uint64_t *empty = codes ? raw_empty : x_empty;
      int stage = 0;
      uint32_t phase = 0;
      uint32_t outstanding = 0, issue_parity = 0;
      const int n_loads = (codes ? n_raw_loads : nkb) + (adapter ? 1 : 0);
      for (int it = 0; it < n_loads; ++it) {
        if (!ptx::mbar_wait(&empty[stage], phase ^ 1, kWaitLimitNs, false)) {
          record_timeout(p.err, abort_flag);
          break;
        }
        const bool main = it < n_loads - (adapter ? 1 : 0);
        if (codes) {
          uint8_t *dst = raw_ring + stage * C::kRawBytes;
          if (main) {
            const int kb = kb0 + it * C::kRawKb;
            ptx::mbar_expect_tx(&full[stage], C::kRawBytes + (p.scale_tma ? C::kScaleBytes : 0));
            ptx::tma_load_2d(dst, &tm_codes, &full[stage], kb * kBK, w0);
            if (p.scale_tma) {
              // scales [N, num_kb]: the aligned group of four k-blocks holding kb, kb + 1
              ptx::tma_load_2d(smem + C::kScaleOff + stage * C::kScaleBytes,
                               &tm_scales, &full[stage], kb & ~3, w0);
            }
          } else {
            // The tile's B^T slice: [128 features, rank] as the A operand.
            ptx::mbar_expect_tx(&full[stage], kBM * p.rank * 2);
            if (p.b_mn) {
              for (int c = 0; c < kBM / 64; ++c) {
                ptx::tma_load_2d(dst + c * (p.rank * 128), &tm_bt, &full[stage], w0 + c * 64, 0);
              }
            } else {
              ptx::tma_load_2d(dst, &tm_bt, &full[stage], 0, w0);
            }
          }
        } else {
          uint8_t *dst = x_ring + stage * C::kXBytes;
          if (main) {
            ptx::mbar_expect_tx(&full[stage], C::kXBytes);
            ptx::tma_load_2d(dst, &tm_x, &full[stage], (kb0 + it) * kBK, 0);
          } else {
            ptx::grid_dep_wait();  // P is the down-projection's output
            ptx::mbar_expect_tx(&full[stage], BT * p.rank * 2);
            ptx::tma_load_2d(dst, &tm_p, &full[stage], 0, 0);
          }
        }
        outstanding |= 1u << stage;
        issue_parity = (issue_parity & ~(1u << stage)) | (phase << stage);
        if (++stage == n_stages) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (aborted(abort_flag)) {
        for (int s = 0; s < n_stages; ++s) {
          if (outstanding & (1u << s)) ptx::mbar_wait(&full[s], (issue_parity >> s) & 1u, 200000000ull);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0 && nkb > 0) {
      const uint32_t idesc = ptx::make_idesc_f16(kBf16, kBM, BT, false, false);
      int xs = 0;
      uint32_t x_phase = 0;
      int c = 0;
      uint32_t c_phase = 0;
      bool ok = true;
      for (int it = 0; it < nkb; ++it) {
        if (!ptx::mbar_wait(&x_full[xs], x_phase, kWaitLimitNs, false) ||
            !ptx::mbar_wait(&conv_full[c], c_phase, kWaitLimitNs, false)) {
          record_timeout(p.err, abort_flag);
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        const uint32_t sa = ptx::smem_addr(conv + c * C::kConvBytes);
        const uint32_t sx = ptx::smem_addr(x_ring + xs * C::kXBytes);
        for (int ks = 0; ks < kBK / kUmmaK; ++ks) {
          ptx::mma_f16(tmem_base, kmajor_desc(sa, 128, ks), kmajor_desc(sx, 128, ks), idesc,
                       (it > 0 || ks > 0) ? 1u : 0u);
        }
        ptx::mma_commit(&x_empty[xs]);
        ptx::mma_commit(&conv_empty[c]);
        if (++xs == C::kXStages) {
          xs = 0;
          x_phase ^= 1;
        }
        if (++c == C::kConvSlots) {
          c = 0;
          c_phase ^= 1;
        }
      }
      if (ok && adapter) {
        // Adapter K-steps: A = B^T slice (next raw slot), B = P (next x slot).
        const int rs = n_raw_loads % C::kRawStages;
        const uint32_t r_phase = static_cast<uint32_t>((n_raw_loads / C::kRawStages) & 1);
        if (!ptx::mbar_wait(&raw_full[rs], r_phase, kWaitLimitNs, false) ||
            !ptx::mbar_wait(&x_full[xs], x_phase, kWaitLimitNs, false)) {
          record_timeout(p.err, abort_flag);
          ok = false;
        } else {
          ptx::tc_fence_after();
          const uint32_t idesc_ad = ptx::make_idesc_f16(kBf16, kBM, BT, p.b_mn != 0, false);
          const uint32_t sa = ptx::smem_addr(raw_ring + rs * C::kRawBytes);
          const uint32_t sx = ptx::smem_addr(x_ring + xs * C::kXBytes);
          const int row_bytes = p.rank * 2;
          for (int ks = 0; ks < p.rank / kUmmaK; ++ks) {
            const uint64_t adesc = p.b_mn ? mnmajor_desc(sa, 128, p.rank * 128, ks)
                                          : kmajor_desc(sa, row_bytes, ks);
            ptx::mma_f16(tmem_base, adesc, kmajor_desc(sx, row_bytes, ks), idesc_ad, 1u);
          }
        }
      }
      if (ok) ptx::mma_commit(tmem_full);
      if (aborted(abort_flag)) {
        ptx::mma_commit(drain);
        ptx::mbar_wait(drain, 0, 200000000ull);
      }
    }
  } else if (warp >= kConvWarp0) {
    // ------------------------------------------------------------------ converters
    // Lane l handles row (group * 8 + l / 4), 16-code chunk l % 4, of the
    // 128 x 64 code tile, writing 32 bytes of the 128B-swizzled bf16 row.
    constexpr int kGroups = kBM / 8 / kConvWarps;  // 2
    // Scales run kScaleAhead k-blocks ahead and each load is issued after the
    // iteration's proxy fence, which would otherwise wait for it.
    constexpr int kScaleAhead = 3;
    const int cw = warp - kConvWarp0;
    const int sub_row = lane / 4;
    const int chunk = lane % 4;
    const float *srow[kGroups];
    float sq[kGroups][kScaleAhead];
#pragma unroll
    for (int g = 0; g < kGroups; ++g) {
      const int n = w0 + (cw + g * kConvWarps) * 8 + sub_row;
      srow[g] = n < p.N && !p.scale_tma
                    ? p.w_scales + static_cast<int64_t>(n) * p.num_kb + kb0 : nullptr;
#pragma unroll
      for (int a = 0; a < kScaleAhead; ++a) {
        sq[g][a] = (srow[g] != nullptr && a < nkb) ? __ldg(srow[g] + a) : 0.0f;
      }
    }
    int rs = 0;
    uint32_t r_phase = 0;
    int c = 0;
    uint32_t c_phase = 0;
    for (int it = 0; it < nkb; ++it) {
      const int sub = it % C::kRawKb;  // k-block within the raw stage
      if (sub == 0 &&
          __any_sync(0xffffffffu, !ptx::mbar_wait(&raw_full[rs], r_phase, kWaitLimitNs, false))) {
        if (lane == 0) record_timeout(p.err, abort_flag);
        break;
      }
      uint4 codes[kGroups];
      const uint8_t *raw = raw_ring + rs * C::kRawBytes;
#pragma unroll
      for (int g = 0; g < kGroups; ++g) {
        // row r's 16-byte chunk j sits at chunk j ^ (r & 7) (TMA 128-byte swizzle)
        const int r = (cw + g * kConvWarps) * 8 + sub_row;
        const int j = (sub * (kBK / 16) + chunk) ^ (r & 7);
        codes[g] = *reinterpret_cast<const uint4 *>(raw + r * (kBK * C::kRawKb) + j * 16);
      }
      if (__any_sync(0xffffffffu,
                     !ptx::mbar_wait(&conv_empty[c], c_phase ^ 1u, kWaitLimitNs, false))) {
        if (lane == 0) record_timeout(p.err, abort_flag);
        break;
      }
      uint8_t *dst = conv + c * C::kConvBytes;
#pragma unroll
      for (int g = 0; g < kGroups; ++g) {
        const int r = (cw + g * kConvWarps) * 8 + sub_row;
        const uint32_t words[4] = {codes[g].x, codes[g].y, codes[g].z, codes[g].w};
        uint32_t outw[8];
        const float sc = p.scale_tma ? scale_ring[rs * (C::kScaleBytes / 4) + r * 4 +
                                                  ((kb0 + it) & 3)]
                                     : sq[g][0];
        const uint64_t sc2 = ptx::splat_f32x2(sc);
#pragma unroll
        for (int wd = 0; wd < 4; ++wd) {
          const uint32_t u = words[wd] ^ 0x80808080u;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            // 2^23 + (q + 128) as floats, then (that - (2^23 + 128)) * s for
            // two codes per packed f32x2 add and multiply: exactly q * s.
            const uint32_t b0 = __byte_perm(u, 0x4B000000u, 0x7440u | (2 * h));
            const uint32_t b1 = __byte_perm(u, 0x4B000000u, 0x7440u | (2 * h + 1));
            float lo, hi;
            ptx::dequant_pair(b0, b1, sc2, lo, hi);
            outw[2 * wd + h] = kBf16 ? ptx::pack_bf16x2(lo, hi) : ptx::pack_f16x2(lo, hi);
          }
        }
        uint8_t *dst_row = dst + r * 128;
        const int sw = r & 7;
        *reinterpret_cast<uint4 *>(dst_row + (((2 * chunk) ^ sw) << 4)) =
            make_uint4(outw[0], outw[1], outw[2], outw[3]);
        *reinterpret_cast<uint4 *>(dst_row + (((2 * chunk + 1) ^ sw) << 4)) =
            make_uint4(outw[4], outw[5], outw[6], outw[7]);
      }
      // The proxy fence orders this warp's generic reads of the raw slot and
      // writes of the converted slot before the TMA refill and the MMA.
      ptx::fence_proxy_async_smem();
      const bool stage_done = sub == C::kRawKb - 1 || it + 1 == nkb;
      if (stage_done) ptx::warp_arrive(&raw_empty[rs]);
      ptx::warp_arrive(&conv_full[c]);
      if (stage_done && ++rs == C::kRawStages) {
        rs = 0;
        r_phase ^= 1;
      }
      if (++c == C::kConvSlots) {
        c = 0;
        c_phase ^= 1;
      }
      if (!p.scale_tma) {
#pragma unroll
        for (int g = 0; g < kGroups; ++g) {
#pragma unroll
          for (int a = 0; a + 1 < kScaleAhead; ++a) sq[g][a] = sq[g][a + 1];
          const int kb = it + kScaleAhead;
          sq[g][kScaleAhead - 1] = (srow[g] != nullptr && kb < nkb) ? __ldg(srow[g] + kb) : 0.0f;
        }
      }
    }
  }

  // ---------------------------------------------------------------- partial tile
  // Every MMA has completed once tmem_full fires, and every ring load was
  // consumed before it, so the rings can hold the fp32 partial.
  if (warp >= kEpiWarp0 && warp < kEpiWarp0 + 4) {
    const int quarter = warp % 4;
    const int row = quarter * 32 + lane;
    bool have = nkb > 0;
    if (have) {
      const bool ok = ptx::mbar_wait(tmem_full, 0, kWaitLimitNs, false);
      if (__any_sync(0xffffffffu, !ok)) {
        if (lane == 0) record_timeout(p.err, abort_flag);
        have = false;
      }
    }
    if (have) ptx::tc_fence_after();
    const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
#pragma unroll 1
    for (int c = 0; c < (BT + 31) / 32; ++c) {
      uint32_t v[32];
      if (have) {
        ptx::tmem_ld_32x32b_x32(t_row + c * 32, v);
        ptx::tmem_ld_wait();
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = 0u;
      }
      float *prow = partial + row * BT + c * 32;
#pragma unroll
      for (int j = 0; j < 32 && c * 32 + j < BT; j += 4) {
        *reinterpret_cast<float4 *>(prow + j) =
            make_float4(__uint_as_float(v[j]), __uint_as_float(v[j + 1]),
                        __uint_as_float(v[j + 2]), __uint_as_float(v[j + 3]));
      }
    }
  }

  // ------------------------------------------------------ cluster reduction
  ptx::tc_fence_before();
  ptx::cluster_sync();
  {
    const int r0 = rank * kBM / p.splits;
    const int r1 = (rank + 1) * kBM / p.splits;
    const int rows = r1 - r0;
    const uint32_t base = ptx::smem_addr(partial);
    for (int item = threadIdx.x; item < rows * (BT / 4); item += C::kThreads) {
      const int row = r0 + item % rows;
      const int t4 = (item / rows) * 4;
      const int n = w0 + row;
      const uint32_t off = static_cast<uint32_t>((row * BT + t4) * 4);
      // Peers' partials are requested four at a time before they are summed.
      float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
      for (int p0 = 0; p0 < 8; p0 += 4) {
        float4 part[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          if (p0 + q < p.splits) {
            part[q] = ptx::ld_shared_cluster_f4(ptx::map_shared_rank(base + off, p0 + q));
          }
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          if (p0 + q < p.splits) {
            acc[0] += part[q].x;
            acc[1] += part[q].y;
            acc[2] += part[q].z;
            acc[3] += part[q].w;
          }
        }
      }
      if (n >= p.N) continue;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int t = t4 + q;
        if (t < p.M) {
          const uint32_t h = kBf16 ? ptx::pack_bf16x2(acc[q], 0.0f) : ptx::pack_f16x2(acc[q], 0.0f);
          p.out[static_cast<int64_t>(t) * p.N + n] = static_cast<uint16_t>(h & 0xffffu);
        }
      }
    }
  }
  // No CTA may leave while a peer can still read its shared memory.
  ptx::cluster_sync();
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem_base, C::kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// W8 + LoRA, swap-AB with 512-token tiles (prefill).
//
// Each converted 128 x 32 weight tile feeds two N = 256 MMAs (tokens
// [t0, t0+256) and [t0+256, t0+512)), so every int8 code is converted once per
// 512 tokens instead of once per 256 (half the conversion work per FLOP of a
// 256-token tile). The 128 x 512 fp32 accumulator takes all 512 TMEM
// columns (single buffer); k-blocks are 32 wide (64-byte swizzled rows) so the
// ring stays 5 stages deep. The adapter runs as rank/16 extra iterations of
// one K = 16 step each (A = 16 columns of B^T, B = 16 columns of P).
// ---------------------------------------------------------------------------
// kBT = 512: one 128 x 512 fp32 accumulator fills TMEM, each converted
// weight tile feeds two N = 256 MMAs. kBT = 256 (the all-gather calls): two
// 128 x 256 accumulators, so a tile's epilogue, whose stores cross NVLink,
// runs while the next tile's main loop fills the other accumulator.
template <bool kTmaStore, int kBT = 512>
struct W8WideCfg {
  static constexpr int BT = kBT;
  static constexpr int kHalves = kBT / 256;            // N = 256 MMAs per k-step
  static constexpr int kAccs = 512 / kBT;              // TMEM accumulators
  static constexpr int kBKw = 32;                      // k-block width (elements)
  static constexpr int kRowBytes = kBKw * 2;           // 64 -> 64-byte swizzle
  static constexpr int kABytes = kBM * kRowBytes;      // 8 KB
  static constexpr int kXHalf = 256 * kRowBytes;       // 16 KB
  static constexpr int kXBytes = kHalves * kXHalf;     // 32 KB (16 KB at kBT = 256)
  static constexpr int kRawBytes = kBM * kBKw;         // 4 KB
  // The stage's scales: 128 rows x the aligned group of four 64-element
  // blocks that holds its k-block (one 16-byte TMA row per feature).
  static constexpr int kScaleBytes = kBM * 4 * 4;      // 2 KB
  // Folded RMSNorm: the stage's 32 norm weights (one 64-byte TMA row; the
  // slot keeps the stage 1 KB-aligned).
  static constexpr int kNormBytes = 1024;
  static constexpr int kStageBytes =
      kABytes + kXBytes + kRawBytes + kScaleBytes + kNormBytes;  // 47 KB (31 KB at kBT 256)
  static constexpr int kStages = kBT == 256 ? 6 : (kTmaStore ? 4 : 5);
  static constexpr int kSlabBytes = 32 * kBM * 2;      // 32 tokens x 128 features, 8 KB
  static constexpr int kStagingBytes = kTmaStore ? 2 * kSlabBytes : 0;
  static constexpr int kThreads = 512;
  static constexpr int kTmemCols = 512;
  static constexpr size_t kSmemBytes =
      1024 + static_cast<size_t>(kStages) * kStageBytes + kStagingBytes + 256;
  static_assert(kStageBytes % 1024 == 0, "stage alignment");
};

// Output tensor maps of the TMA-store epilogue: one per destination, each a
// [M, ldy] 16-bit matrix with 32 x 128 boxes.
struct OutMaps {
  CUtensorMap map[kMaxOuts];
};

template <bool kBf16, bool kTmaStore, int kBT, bool kNorm>
__global__ void __launch_bounds__(W8WideCfg<kTmaStore, kBT>::kThreads, 1)
    w8_wide_kernel(const __grid_constant__ CUtensorMap tm_x,
                   const __grid_constant__ CUtensorMap tm_codes,
                   const __grid_constant__ CUtensorMap tm_p,
                   const __grid_constant__ CUtensorMap tm_bt,
                   const __grid_constant__ CUtensorMap tm_scales,
                   const __grid_constant__ CUtensorMap tm_norm,
                   const __grid_constant__ OutMaps out_maps, const W8Params p) {
  using C = W8WideCfg<kTmaStore, kBT>;
  constexpr int BT = C::BT;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t *staging = smem + C::kStages * C::kStageBytes;
  uint64_t *bars = reinterpret_cast<uint64_t *>(staging + C::kStagingBytes);
  uint64_t *full = bars;
  uint64_t *empty = bars + C::kStages;
  uint64_t *conv_full = bars + 2 * C::kStages;
  uint64_t *tmem_full = bars + 3 * C::kStages;  // [kAccs]
  uint64_t *tmem_empty = tmem_full + C::kAccs;  // [kAccs]
  uint64_t *drain = tmem_empty + C::kAccs;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
  int *abort_flag = reinterpret_cast<int *>(tmem_slot + 1);

  const int warp = threadIdx.x / kWarp;
  const int lane = threadIdx.x % kWarp;
  const int n_extra = p.extra_ksteps;  // one K = 16 iteration per 16 adapter columns
  const int num_iters = p.num_kb + n_extra;

  if (threadIdx.x == 0) {
    // Descriptor fetches overlap the setup instead of the first loads.
    ptx::prefetch_tensor_map(&tm_codes);
    ptx::prefetch_tensor_map(&tm_x);
    ptx::prefetch_tensor_map(&tm_p);
    ptx::prefetch_tensor_map(&tm_bt);
    for (int s = 0; s < C::kStages; ++s) {
      ptx::mbar_init(&full[s], 1);
      ptx::mbar_init(&empty[s], 1);
      ptx::mbar_init(&conv_full[s], kConvThreads / kWarp);
    }
    for (int a = 0; a < C::kAccs; ++a) {
      ptx::mbar_init(&tmem_full[a], 1);
      ptx::mbar_init(&tmem_empty[a], 4);
    }
    ptx::mbar_init(drain, 1);
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == 1) {
    ptx::tmem_alloc(tmem_slot, C::kTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t outstanding = 0, issue_parity = 0;
      bool dep_ready = false;
      for (int tile = blockIdx.x; tile < p.n_tiles && !aborted(abort_flag); tile += gridDim.x) {
        const int w0 = (tile % p.n_tiles_w) * kBM;
        const int t0 = (tile / p.n_tiles_w) * BT;
        for (int it = 0; it < num_iters; ++it) {
          if (!ptx::mbar_wait(&empty[stage], phase ^ 1)) {
            record_timeout(p.err, abort_flag);
            break;
          }
          uint8_t *sa = smem + stage * C::kStageBytes;
          uint8_t *sx = sa + C::kABytes;
          if (it < p.num_kb) {
            const int k0 = it * C::kBKw;
            ptx::mbar_expect_tx(&full[stage], C::kXBytes + C::kRawBytes +
                                                  (p.scale_tma ? C::kScaleBytes : 0) +
                                                  (kNorm ? C::kBKw * 4 : 0));
            if constexpr (kNorm) {
              ptx::tma_load_2d(sx + C::kXBytes + C::kRawBytes + C::kScaleBytes, &tm_norm,
                               &full[stage], k0, 0);
            }
            for (int h = 0; h < C::kHalves; ++h) {
              ptx::tma_load_2d(sx + h * C::kXHalf, &tm_x, &full[stage], k0, t0 + h * 256);
            }
            ptx::tma_load_2d(sx + C::kXBytes, &tm_codes, &full[stage], k0, w0);
            if (p.scale_tma) {
              ptx::tma_load_2d(sx + C::kXBytes + C::kRawBytes, &tm_scales, &full[stage],
                               (it / 2) & ~3, w0);
            }
          } else {
            if (!dep_ready) {  // P comes from the down-projection launched just before
              ptx::grid_dep_wait();
              dep_ready = true;
            }
            const int j0 = (it - p.num_kb) * kUmmaK;  // adapter columns [j0, j0 + 16)
            ptx::mbar_expect_tx(&full[stage], (kBM + BT) * kUmmaK * 2);
            if (p.extra_b_mn) {
              for (int c = 0; c < kBM / 64; ++c) {
                ptx::tma_load_2d(sa + c * (kUmmaK * 128), &tm_bt, &full[stage], w0 + c * 64, j0);
              }
            } else {
              ptx::tma_load_2d(sa, &tm_bt, &full[stage], j0, w0);
            }
            for (int h = 0; h < C::kHalves; ++h) {
              ptx::tma_load_2d(sx + h * C::kXHalf, &tm_p, &full[stage], j0, t0 + h * 256);
            }
          }
          outstanding |= 1u << stage;
          issue_parity = (issue_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (aborted(abort_flag)) {
        for (int s = 0; s < C::kStages; ++s) {
          if (outstanding & (1u << s)) ptx::mbar_wait(&full[s], (issue_parity >> s) & 1u, 200000000ull);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc_main = ptx::make_idesc_f16(kBf16, kBM, 256, false, false);
      const uint32_t idesc_extra = ptx::make_idesc_f16(kBf16, kBM, 256, p.extra_b_mn != 0, false);
      int stage = 0;
      uint32_t phase = 0;
      uint32_t conv_parity = 0;
      int local = 0;
      for (int tile = blockIdx.x; tile < p.n_tiles && !aborted(abort_flag);
           tile += gridDim.x, ++local) {
        const int acc = local % C::kAccs;
        const uint32_t acc_base = tmem_base + acc * 256;
        if (!ptx::mbar_wait(&tmem_empty[acc], static_cast<uint32_t>((local / C::kAccs) & 1) ^ 1u)) {
          record_timeout(p.err, abort_flag);
          break;
        }
        ptx::tc_fence_after();
        bool ok = true;
        for (int it = 0; it < num_iters; ++it) {
          const bool main_kb = it < p.num_kb;
          const uint32_t want = main_kb ? (conv_parity >> stage) & 1u : phase;
          if (main_kb) conv_parity ^= 1u << stage;
          if (!ptx::mbar_wait(main_kb ? &conv_full[stage] : &full[stage], want)) {
            record_timeout(p.err, abort_flag);
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          const uint32_t sa = ptx::smem_addr(smem + stage * C::kStageBytes);
          const uint32_t sx = sa + C::kABytes;
          if (main_kb) {
            for (int ks = 0; ks < C::kBKw / kUmmaK; ++ks) {
              const uint64_t adesc = kmajor_desc(sa, C::kRowBytes, ks);
              for (int h = 0; h < C::kHalves; ++h) {
                ptx::mma_f16(acc_base + h * 256, adesc,
                             kmajor_desc(sx + h * C::kXHalf, C::kRowBytes, ks), idesc_main,
                             (it > 0 || ks > 0) ? 1u : 0u);
              }
            }
          } else {
            const uint64_t adesc = p.extra_b_mn ? mnmajor_desc(sa, 128, kUmmaK * 128, 0)
                                                : kmajor_desc(sa, kUmmaK * 2, 0);
            for (int h = 0; h < C::kHalves; ++h) {
              ptx::mma_f16(acc_base + h * 256, adesc,
                           kmajor_desc(sx + h * C::kXHalf, kUmmaK * 2, 0), idesc_extra,
                           it > 0 ? 1u : 0u);
            }
          }
          ptx::mma_commit(&empty[stage]);
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        ptx::mma_commit(&tmem_full[acc]);
      }
      if (aborted(abort_flag)) {
        ptx::mma_commit(drain);
        ptx::mbar_wait(drain, 0, 200000000ull);
      }
    }
  } else if (warp >= kEpiWarp0 && warp < kEpiWarp0 + 4) {
    // ------------------------------------------------------------------ epilogue
    const int quarter = warp % 4;
    const int row = quarter * 32 + lane;
    uint32_t slab = 0;
    int local = 0;
    for (int tile = blockIdx.x; tile < p.n_tiles; tile += gridDim.x, ++local) {
      const int w0 = (tile % p.n_tiles_w) * kBM;
      const int t0 = (tile / p.n_tiles_w) * BT;
      // With the TMA-store path the four epilogue warps share named barriers,
      // so they decide together whether to go on.
      const int acc = local % C::kAccs;
      bool ok = ptx::warp_wait(&tmem_full[acc], static_cast<uint32_t>((local / C::kAccs) & 1));
      if constexpr (kTmaStore) ok = ptx::named_bar_all(1, 4 * kWarp, ok);
      if (!ok) {
        if (lane == 0) record_timeout(p.err, abort_flag);
        break;
      }
      ptx::tc_fence_after();
      const uint32_t t_row =
          tmem_base + acc * 256 + (static_cast<uint32_t>(quarter * 32) << 16);
      const int n = w0 + row;
      uint16_t *out = static_cast<uint16_t *>(p.outs[0]);
#pragma unroll 1
      for (int c = 0; c < BT / 32; ++c) {
        uint32_t v[32];
        float rs_lane = 1.0f;
        if constexpr (kNorm) {
          const int t = t0 + c * 32 + lane;
          rs_lane = t < p.M ? __ldg(p.row_scale + t) : 0.0f;
        }
        ptx::tmem_ld_32x32b_x32(t_row + c * 32, v);
        ptx::tmem_ld_wait();
        if constexpr (kNorm) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            v[j] = __float_as_uint(__uint_as_float(v[j]) * __shfl_sync(0xffffffffu, rs_lane, j));
          }
        }
        if constexpr (kTmaStore) {
          // Stage a 32-token x 128-feature slab (token-major, 256-byte rows)
          // and let the TMA engine store it to every destination; the slab
          // buffer is double-buffered against the stores still reading it.
          const bool elected = threadIdx.x == kEpiWarp0 * kWarp;
          if (elected) ptx::bulk_wait_read<1>();
          ptx::named_bar_sync(1, 4 * kWarp);
          uint16_t *stg = reinterpret_cast<uint16_t *>(staging + (slab & 1) * C::kSlabBytes);
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const float f = __uint_as_float(v[j]);
            const uint32_t h = kBf16 ? ptx::pack_bf16x2(f, 0.0f) : ptx::pack_f16x2(f, 0.0f);
            stg[j * kBM + row] = static_cast<uint16_t>(h & 0xffffu);
          }
          ptx::fence_proxy_async_smem();
          ptx::named_bar_sync(1, 4 * kWarp);
          if (p.mc_out != nullptr) {
            // One multicast write per 16 bytes reaches every rank's copy: the
            // 128 epilogue threads each send 4 of the slab's 512 chunks
            // (token j, 8 features). The slab buffer is reused two slabs
            // later, after every thread has passed the next barrier.
            const int epi = threadIdx.x - kEpiWarp0 * kWarp;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int q = epi + i * 128;
              const int j = q >> 4;
              const int f8 = (q & 15) * 8;
              const int t = t0 + c * 32 + j;
              if (t < p.M) {
                const uint4 v = *reinterpret_cast<const uint4 *>(stg + j * kBM + f8);
                uint16_t *dst = static_cast<uint16_t *>(p.mc_out) +
                                static_cast<int64_t>(t) * p.ldo + p.out_col0 + w0 + f8;
                ptx::multimem_st_v4(dst, v);
              }
            }
          } else if (elected) {
            // The local copy first, then the peers (NVLink).
            ptx::tma_store_2d(&out_maps.map[p.self_out], stg, p.out_col0 + w0, t0 + c * 32);
            for (int d = 0; d < p.n_outs; ++d) {
              if (d != p.self_out) ptx::tma_store_2d(&out_maps.map[d], stg, p.out_col0 + w0, t0 + c * 32);
            }
            ptx::bulk_commit();
          }
          ++slab;
        } else if (n < p.N) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int t = t0 + c * 32 + j;
            if (t < p.M) {
              const float f = __uint_as_float(v[j]);
              const uint32_t h = kBf16 ? ptx::pack_bf16x2(f, 0.0f) : ptx::pack_f16x2(f, 0.0f);
              out[static_cast<int64_t>(t) * p.ldo + p.out_col0 + n] =
                  static_cast<uint16_t>(h & 0xffffu);
            }
          }
        }
      }
      ptx::tc_fence_before();
      ptx::warp_arrive(&tmem_empty[acc]);
      if constexpr (kTmaStore) {
        if (p.done != nullptr && threadIdx.x == kEpiWarp0 * kWarp) {
          // Publish the tile: its stores have completed (not just read
          // shared memory) before the group counter moves.
          ptx::bulk_wait_all();
          ptx::fence_proxy_async_global();
          __threadfence();
          atomicAdd(p.done + (t0 / BT) / p.rb_per_group, 1u);
        }
      }
    }
    if constexpr (kTmaStore) {
      // Stores must finish reading shared memory before the CTA exits.
      if (threadIdx.x == kEpiWarp0 * kWarp) ptx::bulk_wait_all();
      if (p.mc_out != nullptr) __threadfence_system();
    }
  } else if (warp >= kConvWarp0) {
    // ------------------------------------------------------------------ converters
    // Lane l of converter warp cw: row cw * 16 + l / 2, 16-code half l % 2 of
    // the 32-code row; writes 32 bytes of the 64-byte swizzled bf16 row
    // (logical 16-byte chunk c sits at c ^ ((row >> 1) & 3)).
    const int cw = warp - kConvWarp0;
    const int r = cw * 16 + lane / 2;
    const int half = lane & 1;
    int stage = 0;
    uint32_t phase = 0;
    for (int tile = blockIdx.x; tile < p.n_tiles; tile += gridDim.x) {
      const int w0 = (tile % p.n_tiles_w) * kBM;
      const int n = w0 + r;
      const float *srow = n < p.N && !p.scale_tma
                              ? p.w_scales + static_cast<int64_t>(n) * p.kb_per_row : nullptr;
      float s_cur = srow != nullptr ? __ldg(srow) : 0.0f;
      bool ok = true;
      for (int it = 0; it < num_iters; ++it) {
        if (it < p.num_kb) {
          const float s_next =
              (srow != nullptr && it + 1 < p.num_kb) ? __ldg(srow + (it + 1) / 2) : 0.0f;
          const bool got = ptx::mbar_wait(&full[stage], phase);
          if (__any_sync(0xffffffffu, !got)) {
            if (lane == 0) record_timeout(p.err, abort_flag);
            ok = false;
            break;
          }
          uint8_t *sa = smem + stage * C::kStageBytes;
          const uint8_t *raw = sa + C::kABytes + C::kXBytes;
          if (p.scale_tma) {
            s_cur = reinterpret_cast<const float *>(raw + C::kRawBytes)[r * 4 + ((it / 2) & 3)];
          }
          const uint4 codes = *reinterpret_cast<const uint4 *>(raw + r * C::kBKw + half * 16);
          const uint32_t words[4] = {codes.x, codes.y, codes.z, codes.w};
          const uint64_t sc2 = ptx::splat_f32x2(s_cur);
          // kNorm: the fp32 norm weights of this lane's 16 input features
          const uint64_t *wsrc = reinterpret_cast<const uint64_t *>(
              raw + C::kRawBytes + C::kScaleBytes + half * 64);
          uint32_t outw[8];
#pragma unroll
          for (int wd = 0; wd < 4; ++wd) {
            const uint32_t u = words[wd] ^ 0x80808080u;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const uint32_t b0 = __byte_perm(u, 0x4B000000u, 0x7440u | (2 * h));
              const uint32_t b1 = __byte_perm(u, 0x4B000000u, 0x7440u | (2 * h + 1));
              float lo, hi;
              if constexpr (kNorm) {
                // code * (block scale * norm weight), rounded once to the dtype
                ptx::dequant_pair(b0, b1, ptx::mul_f32x2(sc2, wsrc[2 * wd + h]), lo, hi);
              } else {
                ptx::dequant_pair(b0, b1, sc2, lo, hi);
              }
              outw[2 * wd + h] = kBf16 ? ptx::pack_bf16x2(lo, hi) : ptx::pack_f16x2(lo, hi);
            }
          }
          uint8_t *dst_row = sa + r * C::kRowBytes;
          const int sw = (r >> 1) & 3;
          *reinterpret_cast<uint4 *>(dst_row + (((2 * half) ^ sw) << 4)) =
              make_uint4(outw[0], outw[1], outw[2], outw[3]);
          *reinterpret_cast<uint4 *>(dst_row + (((2 * half + 1) ^ sw) << 4)) =
              make_uint4(outw[4], outw[5], outw[6], outw[7]);
          ptx::fence_proxy_async_smem();
          ptx::warp_arrive(&conv_full[stage]);
          s_cur = s_next;
        } else if (!ptx::mbar_wait(&full[stage], phase)) {
          // Adapter stages are not converted, but waiting for them keeps this
          // warp within one phase of every stage's barrier (a parity wait
          // cannot tell phase u from phase u - 2).
          if (lane == 0) record_timeout(p.err, abort_flag);
          ok = false;
          break;
        }
        if (++stage == C::kStages) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (!ok) break;
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem_base, C::kTmemCols);
  }
  if (p.done != nullptr && threadIdx.x == 0 && aborted(abort_flag)) {
    // This CTA gave up on some tiles: push every counter past its target so
    // that copies waiting on them are released (the error word says the
    // output is invalid).
    for (int g = 0; g < p.n_groups; ++g) atomicAdd(p.done + g, 1u << 24);
  }
}

// ---------------------------------------------------------------------------
// fp32 LoRA linear on the tensor cores: kind::tf32 with a three-product split.
//
// The reference's CUDA lora_linear is fp32 (cpp/src/bindings.cpp:94-127,
// cuda/src/lora_linear.cu:237-277, CUDA-core FMA); its tests hold it to 1e-3
// of an fp32 CPU product. One tf32 pass (10 explicit mantissa bits) is not
// that accurate, so every operand v is split into hi = tf32(v) and
// lo = v - hi (exact in fp32) and the MMA accumulates hi*hi + hi*lo + lo*hi in
// fp32; the dropped lo*lo term is below 2^-22 of the product.
//
// One kernel serves both launches of a call: the down-projection (B = A_lora,
// N = rank, out = P scaled by alpha/r) and the main product, whose adapter is
// ceil(rank/32) extra k-blocks with A = P tile and B = the B_lora slice. The
// splitters write hi over the loaded tile and lo into a twin buffer 16 KB
// above it, both K-major (128-byte rows of 32 k, 128B-swizzled), which is the
// only operand form the MMA is given. A B operand stored [K, N] (N
// contiguous) arrives as four 32-column x 32-row chunks and is transposed by
// the splitters in 4 x 4 register blocks on the way.
//   warp 0 TMA producer, warp 1 TMEM owner + MMA issuer, warps 4-7 epilogue
//   (thread = output row), warps 8-15 splitters; 128 x 128 tiles, persistent,
//   double-buffered TMEM accumulators.
// ---------------------------------------------------------------------------
struct F32Cfg {
  static constexpr int BN = 128;
  static constexpr int kBKf = 32;                      // k-block: 32 fp32 = one 128 B row
  static constexpr int kTileBytes = 128 * kBKf * 4;    // 16 KB (A or B, hi or lo)
  static constexpr int kStageBytes = 4 * kTileBytes;   // A hi, A lo, B hi, B lo
  static constexpr int kStages = 3;
  static constexpr int kThreads = 512;
  static constexpr int kTmemCols = 2 * BN;
  static constexpr size_t kSmemBytes = 1024 + static_cast<size_t>(kStages) * kStageBytes + 256;
};

struct F32Params {
  int M, N;
  int num_kb;       // main k-blocks (ceil(K / 32))
  int extra_kb;     // adapter k-blocks (ceil(rank / 32)); 0 for the down-projection
  int n_mma;        // MMA N (16..128, multiple of 16)
  int b_mn;         // main B stored [K, N]
  int e_mn;         // adapter B stored [rank, N]
  int ldo;          // output row stride (elements)
  int products;     // 3: hi*hi + hi*lo + lo*hi (fp32 accuracy); 1: hi*hi (tf32)
  float out_scale;
  float *out;       // [M, ldo] fp32
  int n_tiles_n;
  int n_tiles_m;
  int band_m;       // row blocks per band of the tile walk (band_order)
  int n_tiles;
  unsigned *err;
};

__global__ void __launch_bounds__(F32Cfg::kThreads, 1)
    lora_f32_kernel(const __grid_constant__ CUtensorMap tm_a,
                    const __grid_constant__ CUtensorMap tm_b,
                    const __grid_constant__ CUtensorMap tm_pa,
                    const __grid_constant__ CUtensorMap tm_pb, const F32Params p) {
  using C = F32Cfg;
  // A second launch that consumes this one's output (P) may start now; it
  // waits for this grid before its first read of P.
  ptx::grid_dep_launch_dependents();
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::kStages * C::kStageBytes);
  uint64_t *full = bars;                        // [kStages] TMA -> splitters
  uint64_t *split = bars + C::kStages;          // [kStages] splitters -> MMA
  uint64_t *empty = bars + 2 * C::kStages;      // [kStages] MMA -> producer
  uint64_t *tmem_full = bars + 3 * C::kStages;  // [2] MMA -> epilogue
  uint64_t *tmem_empty = tmem_full + 2;         // [2] epilogue -> MMA
  uint64_t *drain = tmem_empty + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
  int *abort_flag = reinterpret_cast<int *>(tmem_slot + 1);
  constexpr int kSplitWarps = kConvThreads / kWarp;

  const int warp = threadIdx.x / kWarp;
  const int lane = threadIdx.x % kWarp;
  const int num_iters = p.num_kb + p.extra_kb;

  if (threadIdx.x == 0) {
    // Descriptor fetches overlap the setup instead of the first loads.
    ptx::prefetch_tensor_map(&tm_a);
    ptx::prefetch_tensor_map(&tm_b);
    ptx::prefetch_tensor_map(&tm_pa);
    ptx::prefetch_tensor_map(&tm_pb);
    for (int s = 0; s < C::kStages; ++s) {
      ptx::mbar_init(&full[s], 1);
      ptx::mbar_init(&split[s], kSplitWarps);
      ptx::mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      ptx::mbar_init(&tmem_full[a], 1);
      ptx::mbar_init(&tmem_empty[a], 4);
    }
    ptx::mbar_init(drain, 1);
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == 1) {
    ptx::tmem_alloc(tmem_slot, C::kTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t outstanding = 0, issue_parity = 0;
      bool dep_ready = false;
      for (int tile = blockIdx.x; tile < p.n_tiles && !aborted(abort_flag); tile += gridDim.x) {
        int mb, nb;
        band_order(tile, p.n_tiles_m, p.n_tiles_n, p.band_m, mb, nb);
        const int m0 = mb * 128;
        const int n0 = nb * C::BN;
        for (int it = 0; it < num_iters; ++it) {
          if (!ptx::mbar_wait(&empty[stage], phase ^ 1)) {
            record_timeout(p.err, abort_flag);
            break;
          }
          uint8_t *sa = smem + stage * C::kStageBytes;
          uint8_t *sb = sa + 2 * C::kTileBytes;
          const bool main_kb = it < p.num_kb;
          if (!main_kb && !dep_ready) {  // P comes from the launch just before
            ptx::grid_dep_wait();
            dep_ready = true;
          }
          const CUtensorMap *ma = main_kb ? &tm_a : &tm_pa;
          const CUtensorMap *mb = main_kb ? &tm_b : &tm_pb;
          const bool mn = main_kb ? p.b_mn != 0 : p.e_mn != 0;
          const int k0 = (main_kb ? it : it - p.num_kb) * C::kBKf;
          ptx::mbar_expect_tx(&full[stage], 2 * C::kTileBytes);
          ptx::tma_load_2d(sa, ma, &full[stage], k0, m0);
          if (mn) {
            // [K, N]: four 32-column chunks of 32 k-rows, 128B-swizzled.
            for (int c = 0; c < C::BN / 32; ++c) {
              ptx::tma_load_2d(sb + c * 4096, mb, &full[stage], n0 + c * 32, k0);
            }
          } else {
            ptx::tma_load_2d(sb, mb, &full[stage], k0, n0);
          }
          outstanding |= 1u << stage;
          issue_parity = (issue_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (aborted(abort_flag)) {
        for (int s = 0; s < C::kStages; ++s) {
          if (outstanding & (1u << s)) ptx::mbar_wait(&full[s], (issue_parity >> s) & 1u, 200000000ull);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = ptx::make_idesc_tf32(128, p.n_mma, false, false);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      for (int tile = blockIdx.x; tile < p.n_tiles && !aborted(abort_flag);
           tile += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = static_cast<uint32_t>((local >> 1) & 1);
        if (!ptx::mbar_wait(&tmem_empty[acc], acc_phase ^ 1)) {
          record_timeout(p.err, abort_flag);
          break;
        }
        ptx::tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * C::BN;
        bool ok = true;
        for (int it = 0; it < num_iters; ++it) {
          if (!ptx::mbar_wait(&split[stage], phase)) {
            record_timeout(p.err, abort_flag);
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          const uint32_t a_hi = ptx::smem_addr(smem + stage * C::kStageBytes);
          const uint32_t a_lo = a_hi + C::kTileBytes;
          const uint32_t b_hi = a_hi + 2 * C::kTileBytes;
          const uint32_t b_lo = a_hi + 3 * C::kTileBytes;
          for (int ks = 0; ks < C::kBKf / 8; ++ks) {
            // K = 8 per MMA: 32 bytes along the 128-byte K-major rows.
            const uint64_t ah = kmajor_desc(a_hi, 128, ks);
            const uint64_t al = kmajor_desc(a_lo, 128, ks);
            const uint64_t bh = kmajor_desc(b_hi, 128, ks);
            const uint64_t bl = kmajor_desc(b_lo, 128, ks);
            const uint32_t first = (it == 0 && ks == 0) ? 0u : 1u;
            ptx::mma_tf32(d_tmem, ah, bh, idesc, first);
            if (p.products == 3) {
              ptx::mma_tf32(d_tmem, ah, bl, idesc, 1u);
              ptx::mma_tf32(d_tmem, al, bh, idesc, 1u);
            }
          }
          ptx::mma_commit(&empty[stage]);
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        ptx::mma_commit(&tmem_full[acc]);
      }
      if (aborted(abort_flag)) {
        ptx::mma_commit(drain);
        ptx::mbar_wait(drain, 0, 200000000ull);
      }
    }
  } else if (warp >= kEpiWarp0 && warp < kEpiWarp0 + 4) {
    // ------------------------------------------------------------------ epilogue
    const int quarter = warp % 4;
    int local = 0;
    for (int tile = blockIdx.x; tile < p.n_tiles; tile += gridDim.x, ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = static_cast<uint32_t>((local >> 1) & 1);
      const bool ok = ptx::warp_wait(&tmem_full[acc], acc_phase);
      if (__any_sync(0xffffffffu, !ok)) {
        if (lane == 0) record_timeout(p.err, abort_flag);
        break;
      }
      ptx::tc_fence_after();
      int mb, nb;
      band_order(tile, p.n_tiles_m, p.n_tiles_n, p.band_m, mb, nb);
      const int m0 = mb * 128;
      const int n0 = nb * C::BN;
      const int row = m0 + quarter * 32 + lane;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * C::BN;
      float *out_row = p.out + static_cast<int64_t>(row) * p.ldo;
#pragma unroll 1
      for (int c = 0; c < p.n_mma / 16; ++c) {
        uint32_t v[32];
        ptx::tmem_ld_32x32b_x16(t_row + c * 16, v);
        ptx::tmem_ld_wait();
        if (row < p.M) {
          const int col0 = n0 + c * 16;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            if (col0 + q * 4 < p.N) {
              *reinterpret_cast<float4 *>(out_row + col0 + q * 4) =
                  make_float4(__uint_as_float(v[4 * q]) * p.out_scale,
                              __uint_as_float(v[4 * q + 1]) * p.out_scale,
                              __uint_as_float(v[4 * q + 2]) * p.out_scale,
                              __uint_as_float(v[4 * q + 3]) * p.out_scale);
            }
          }
        }
      }
      ptx::tc_fence_before();
      ptx::warp_arrive(&tmem_empty[acc]);
    }
  } else if (warp >= kConvWarp0) {
    // ------------------------------------------------------------------ splitters
    // A tile (and a K-major B tile): thread t splits float4 q = i * 256 + t
    // in place (hi) and 16 KB above (lo); the swizzle is the same for both.
    // An MN-major B tile: thread t owns the 4 x 4 block at n = 4 (t % 32),
    // k = 4 (t / 32), reads it from its chunk, and after all splitters have
    // read, writes it transposed as four 16-byte K-major row pieces.
    // A warp whose wait gives up (or that sees another role give up) switches
    // to abort mode: it skips waits and work but still takes part in every
    // named barrier the other splitters will reach, so none can wait forever.
    const int t = threadIdx.x - kConvWarp0 * kWarp;
    int stage = 0;
    uint32_t phase = 0;
    bool abort_mode = false;
    for (int tile = blockIdx.x; tile < p.n_tiles; tile += gridDim.x) {
      for (int it = 0; it < num_iters; ++it) {
        if (!abort_mode) {
          if (__any_sync(0xffffffffu, !ptx::mbar_wait(&full[stage], phase))) {
            if (lane == 0) record_timeout(p.err, abort_flag);
            abort_mode = true;
          } else if (aborted(abort_flag)) {
            abort_mode = true;
          }
        }
        uint8_t *base = smem + stage * C::kStageBytes;
        const bool mn = it < p.num_kb ? p.b_mn != 0 : p.e_mn != 0;
        const int n_flat = mn ? 4 : 8;  // float4s split element-wise per thread
        if (!abort_mode) {
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            if (i >= n_flat) break;
            const int q = i * kConvThreads + t;  // A: 0..1023, B (K-major): 1024..2047
            uint8_t *hi = base + (q >> 10) * 2 * C::kTileBytes + (q & 1023) * 16;
            const float4 v = *reinterpret_cast<float4 *>(hi);
            float4 h, l;
            h.x = ptx::round_tf32(v.x); l.x = v.x - h.x;
            h.y = ptx::round_tf32(v.y); l.y = v.y - h.y;
            h.z = ptx::round_tf32(v.z); l.z = v.z - h.z;
            h.w = ptx::round_tf32(v.w); l.w = v.w - h.w;
            *reinterpret_cast<float4 *>(hi) = h;
            *reinterpret_cast<float4 *>(hi + C::kTileBytes) = l;
          }
        }
        if (mn) {
          uint8_t *bt = base + 2 * C::kTileBytes;
          const int n0 = 4 * (t % 32);
          const int k0 = 4 * (t / 32);
          const int chunk = n0 / 32;
          const int j = (n0 % 32) / 4;  // 16-byte column of the chunk row
          const bool work = !abort_mode;
          float blk[4][4];              // [k][n]
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const int k = k0 + kk;
            float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            if (work) {
              v = *reinterpret_cast<const float4 *>(bt + chunk * 4096 + k * 128 +
                                                    ((j ^ (k & 7)) << 4));
            }
            blk[kk][0] = v.x;
            blk[kk][1] = v.y;
            blk[kk][2] = v.z;
            blk[kk][3] = v.w;
          }
          ptx::named_bar_sync(2, kConvThreads);  // every chunk read before any row is written
          if (work) {
#pragma unroll
            for (int nn = 0; nn < 4; ++nn) {
              const int n = n0 + nn;
              float4 h, l;
              h.x = ptx::round_tf32(blk[0][nn]); l.x = blk[0][nn] - h.x;
              h.y = ptx::round_tf32(blk[1][nn]); l.y = blk[1][nn] - h.y;
              h.z = ptx::round_tf32(blk[2][nn]); l.z = blk[2][nn] - h.z;
              h.w = ptx::round_tf32(blk[3][nn]); l.w = blk[3][nn] - h.w;
              uint8_t *dst = bt + n * 128 + (((k0 / 4) ^ (n & 7)) << 4);
              *reinterpret_cast<float4 *>(dst) = h;
              *reinterpret_cast<float4 *>(dst + C::kTileBytes) = l;
            }
          }
        }
        if (!abort_mode) {
          ptx::fence_proxy_async_smem();
          ptx::warp_arrive(&split[stage]);
        }
        if (++stage == C::kStages) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem_base, C::kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// LoRA merge + block-INT8 quantisation in one pass:
//   codes, scales = quantize_int8(W + scaling * (lora_b @ lora_a))
// with the module's layouts (training/lora.py:95-102: W [out, in], lora_a
// [rank, in], lora_b [out, rank]) and 16-bit W, lora_a, lora_b.
//
// The rank-r product is a tcgen05 MMA per 128-row x 256-column tile of W
// (A operand = lora_b rows, K-major; B operand = lora_a, MN-major in 64-column
// chunks; K = rank), accumulated in TMEM. The epilogue thread owns one row of
// W, so each 64-element quantisation block is 64 consecutive accumulator
// columns of one thread: it rounds like the module's dtype does (the product
// to the dtype, times scaling to the dtype, plus W to the dtype), takes the
// block absmax with no cross-thread reduction, and writes the codes and the
// scale with the quantiser's exact arithmetic. The W tile arrives by TMA in
// the same stage (128B-swizzled 64-column boxes, so a warp's row reads spread
// over the banks); a stage is released once the MMA and every epilogue warp
// are done with it. W is read once and the merged weight never reaches memory.
//   warp 0 TMA producer, warp 1 TMEM owner + MMA issuer, warps 4-19 epilogue.
// ---------------------------------------------------------------------------
struct MergeCfg {
  static constexpr int BK = 256;                         // columns of W per tile
  static constexpr int kBBytes = kBM * 64 * 2;            // lora_b rows, rank <= 64
  static constexpr int kABytes = 64 * BK * 2;             // lora_a columns, rank <= 64
  static constexpr int kWBytes = kBM * BK * 2;            // W tile: 4 boxes of 128 x 64
  static constexpr int kStageBytes = kBBytes + kABytes + kWBytes;  // 112 KB
  // Two stages fill shared memory, which also keeps one CTA per SM: the two
  // 256-column accumulators take all of an SM's TMEM.
  static constexpr int kStages = 2;
  // Sixteen epilogue warps (warps 4-19), four per TMEM lane quarter, each
  // taking one of a tile's four 64-column blocks: the per-element merge and
  // quantise work needs several warps per scheduler to hide its latency.
  static constexpr int kEpiWarps = 16;
  static constexpr int kThreads = (kEpiWarp0 + kEpiWarps) * kWarp;
  static constexpr int kTmemCols = 2 * BK;
  static constexpr size_t kSmemBytes = 1024 + static_cast<size_t>(kStages) * kStageBytes + 256;
};

struct MergeParams {
  int N, K;              // W is [N, K]
  int rank;
  float scaling;
  const uint16_t *w;
  int8_t *codes;         // [N, K]
  float *scales;         // [N, K / 64]
  int n_tiles_k;
  int n_tiles;
  unsigned *err;
};

// Two floats rounded to the 16-bit storage type and back (one packed
// conversion for the pair).
template <bool kBf16>
__device__ __forceinline__ void round_pair(float &lo, float &hi) {
  if constexpr (kBf16) {
    const uint32_t h = ptx::pack_bf16x2(lo, hi);
    lo = __uint_as_float(h << 16);
    hi = __uint_as_float(h & 0xffff0000u);
  } else {
    const float2 f = __half22float2(__halves2half2(__float2half_rn(lo), __float2half_rn(hi)));
    lo = f.x;
    hi = f.y;
  }
}

// The two 16-bit values of a word as floats.
template <bool kBf16>
__device__ __forceinline__ void unpack_pair(uint32_t w, float &lo, float &hi) {
  if constexpr (kBf16) {
    lo = __uint_as_float(w << 16);
    hi = __uint_as_float(w & 0xffff0000u);
  } else {
    const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&w));
    lo = f.x;
    hi = f.y;
  }
}

template <bool kBf16>
__global__ void __launch_bounds__(MergeCfg::kThreads, 1)
    lora_merge_quant_kernel(const __grid_constant__ CUtensorMap tm_b,
                            const __grid_constant__ CUtensorMap tm_a,
                            const __grid_constant__ CUtensorMap tm_w, const MergeParams p) {
  using C = MergeCfg;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::kStages * C::kStageBytes);
  uint64_t *full = bars;
  uint64_t *empty = bars + C::kStages;
  uint64_t *tmem_full = bars + 2 * C::kStages;
  uint64_t *tmem_empty = tmem_full + 2;
  uint64_t *drain = tmem_empty + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
  int *abort_flag = reinterpret_cast<int *>(tmem_slot + 1);

  const int warp = threadIdx.x / kWarp;
  const int lane = threadIdx.x % kWarp;

  if (threadIdx.x == 0) {
    // Descriptor fetches overlap the setup instead of the first loads.
    ptx::prefetch_tensor_map(&tm_b);
    ptx::prefetch_tensor_map(&tm_a);
    ptx::prefetch_tensor_map(&tm_w);
    for (int s = 0; s < C::kStages; ++s) {
      ptx::mbar_init(&full[s], 1);
      ptx::mbar_init(&empty[s], 1 + C::kEpiWarps);  // MMA commit + epilogue warps
    }
    for (int a = 0; a < 2; ++a) {
      ptx::mbar_init(&tmem_full[a], 1);
      ptx::mbar_init(&tmem_empty[a], C::kEpiWarps);
    }
    ptx::mbar_init(drain, 1);
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == 1) {
    ptx::tmem_alloc(tmem_slot, C::kTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t outstanding = 0, issue_parity = 0;
      for (int tile = blockIdx.x; tile < p.n_tiles && !aborted(abort_flag); tile += gridDim.x) {
        const int n0 = (tile / p.n_tiles_k) * kBM;
        const int k0 = (tile % p.n_tiles_k) * C::BK;
        if (!ptx::mbar_wait(&empty[stage], phase ^ 1)) {
          record_timeout(p.err, abort_flag);
          break;
        }
        uint8_t *sb = smem + stage * C::kStageBytes;
        uint8_t *sa = sb + C::kBBytes;
        uint8_t *sw = sa + C::kABytes;
        ptx::mbar_expect_tx(&full[stage], (kBM + C::BK) * p.rank * 2 + C::kWBytes);
        ptx::tma_load_2d(sb, &tm_b, &full[stage], 0, n0);
        for (int c = 0; c < C::BK / 64; ++c) {
          ptx::tma_load_2d(sa + c * (p.rank * 128), &tm_a, &full[stage], k0 + c * 64, 0);
          ptx::tma_load_2d(sw + c * (kBM * 128), &tm_w, &full[stage], k0 + c * 64, n0);
        }
        outstanding |= 1u << stage;
        issue_parity = (issue_parity & ~(1u << stage)) | (phase << stage);
        if (++stage == C::kStages) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (aborted(abort_flag)) {
        for (int s = 0; s < C::kStages; ++s) {
          if (outstanding & (1u << s)) ptx::mbar_wait(&full[s], (issue_parity >> s) & 1u, 200000000ull);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = ptx::make_idesc_f16(kBf16, kBM, C::BK, false, true);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      for (int tile = blockIdx.x; tile < p.n_tiles && !aborted(abort_flag);
           tile += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = static_cast<uint32_t>((local >> 1) & 1);
        if (!ptx::mbar_wait(&tmem_empty[acc], acc_phase ^ 1) ||
            !ptx::mbar_wait(&full[stage], phase)) {
          record_timeout(p.err, abort_flag);
          break;
        }
        ptx::tc_fence_after();
        const uint32_t sb = ptx::smem_addr(smem + stage * C::kStageBytes);
        const uint32_t sa = sb + C::kBBytes;
        for (int ks = 0; ks < p.rank / kUmmaK; ++ks) {
          ptx::mma_f16(tmem_base + acc * C::BK, kmajor_desc(sb, p.rank * 2, ks),
                       mnmajor_desc(sa, 128, p.rank * 128, ks), idesc, ks > 0 ? 1u : 0u);
        }
        ptx::mma_commit(&empty[stage]);
        ptx::mma_commit(&tmem_full[acc]);
        if (++stage == C::kStages) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (aborted(abort_flag)) {
        ptx::mma_commit(drain);
        ptx::mbar_wait(drain, 0, 200000000ull);
      }
    }
  } else if (warp >= kEpiWarp0 && warp < kEpiWarp0 + C::kEpiWarps) {
    // ------------------------------------------------------------------ epilogue
    const int quarter = warp % 4;
    const int blk = (warp - kEpiWarp0) / 4;  // this warp's 64-column block of every tile
    int local = 0;
    for (int tile = blockIdx.x; tile < p.n_tiles; tile += gridDim.x, ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = static_cast<uint32_t>((local >> 1) & 1);
      const bool ok = ptx::warp_wait(&tmem_full[acc], acc_phase);
      if (__any_sync(0xffffffffu, !ok)) {
        if (lane == 0) record_timeout(p.err, abort_flag);
        break;
      }
      ptx::tc_fence_after();
      const int row = quarter * 32 + lane;
      const int n = (tile / p.n_tiles_k) * kBM + row;
      const int kb = (tile % p.n_tiles_k) * C::BK + blk * 64;
      const int stage = local % C::kStages;  // one stage per tile
      const uint8_t *wrow = smem + stage * C::kStageBytes + C::kBBytes + C::kABytes +
                            blk * (kBM * 128) + row * 128;
      const uint32_t t_col = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                             acc * C::BK + blk * 64;
      if (kb < p.K) {  // warp-uniform
        // Merged values, rounded to the storage type, kept packed two per word.
        uint32_t mw[32];
        unsigned amax = 0;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          uint32_t v[32];
          ptx::tmem_ld_32x32b_x32(t_col + half * 32, v);
          ptx::tmem_ld_wait();
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int chunk = half * 4 + q;  // 16-byte chunk of the 128-byte row
            const uint4 wv = *reinterpret_cast<const uint4 *>(wrow + ((chunk ^ (row & 7)) << 4));
            const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
            for (int h = 0; h < 4; ++h) {
              const int e = q * 8 + 2 * h;  // within this half
              // As the module computes it in its dtype: the product rounded,
              // scaled and rounded, added to W and rounded.
              float p0 = __uint_as_float(v[e]), p1 = __uint_as_float(v[e + 1]);
              round_pair<kBf16>(p0, p1);
              float u0 = p0 * p.scaling, u1 = p1 * p.scaling;
              round_pair<kBf16>(u0, u1);
              float w0, w1;
              unpack_pair<kBf16>(ww[h], w0, w1);
              const float m0 = w0 + u0, m1 = w1 + u1;
              const uint32_t packed = kBf16 ? ptx::pack_bf16x2(m0, m1) : ptx::pack_f16x2(m0, m1);
              mw[half * 16 + q * 4 + h] = packed;
              float r0, r1;
              unpack_pair<kBf16>(packed, r0, r1);
              amax = max(amax, max(__float_as_uint(r0) & 0x7fffffffu,
                                   __float_as_uint(r1) & 0x7fffffffu));
            }
          }
        }
        if (n < p.N) {
          const float s = block_scale(amax);
          const bool fast = quotient_path_ok(amax, s);
          const float r = __frcp_rn(s);
          uint4 *dst = reinterpret_cast<uint4 *>(p.codes + static_cast<int64_t>(n) * p.K + kb);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint32_t words[4];
#pragma unroll
            for (int w4 = 0; w4 < 4; ++w4) {
              float x0, x1, x2, x3;
              unpack_pair<kBf16>(mw[q * 8 + 2 * w4], x0, x1);
              unpack_pair<kBf16>(mw[q * 8 + 2 * w4 + 1], x2, x3);
              const float xs[4] = {x0, x1, x2, x3};
              uint32_t word = 0;
#pragma unroll
              for (int b4 = 0; b4 < 4; ++b4) {
                const uint32_t cb = fast ? code_bits_fast(xs[b4], s, r) : code_bits_exact(xs[b4], s);
                word |= (cb & 0xffu) << (8 * b4);
              }
              words[w4] = word;
            }
            dst[q] = make_uint4(words[0], words[1], words[2], words[3]);
          }
          p.scales[static_cast<int64_t>(n) * (p.K / 64) + kb / 64] = s;
        }
      }
      ptx::tc_fence_before();
      ptx::warp_arrive(&tmem_empty[acc]);
      ptx::warp_arrive(&empty[stage]);  // this warp's W reads are done
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem_base, C::kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// W8 gate and up projections of a LLaMA MLP with the SwiGLU fused into the
// epilogue (the reference's examples/transformer_block.py:70-89 computes
// swiglu(gate(x), up(x)), and its cuda/src/activations.cu:19-21, 68-76
// defines silu(x) = x / (1 + exp(-x))):
//   h[t, f] = silu(g) * u,  g = round(x Wg^T)[t, f],  u = round(x Wu^T)[t, f]
// with g and u rounded to the activation dtype as the two projections' outputs
// would be, and h computed in fp32 and rounded once.
//
// Swap-AB like w8_wide_kernel: a tile is 128 features x 256 tokens; each stage
// carries the gate and the up code tiles of the same 128 features (32-wide
// k-blocks) and one activation tile, the converters turn both into bf16/f16,
// and per k-step two N = 256 MMAs accumulate g into TMEM columns 0-255 and u
// into 256-511 against the same activation operand. The epilogue thread owns
// feature row f of both accumulators, so silu(g) * u needs no exchange; the
// result goes out through the staged TMA-store path. Only h reaches memory.
//   warp 0 TMA producer, warp 1 TMEM owner + MMA issuer, warps 4-7 epilogue,
//   warps 8-23 converters.
// ---------------------------------------------------------------------------
struct SwigluCfg {
  static constexpr int BT = 256;                       // tokens per tile
  static constexpr int kBKw = 32;                      // k-block width
  static constexpr int kRowBytes = kBKw * 2;           // 64 -> 64-byte swizzle
  static constexpr int kABytes = kBM * kRowBytes;      // 8 KB per converted tile
  static constexpr int kXBytes = BT * kRowBytes;       // 16 KB
  static constexpr int kRawBytes = kBM * kBKw;         // 4 KB per code tile
  // [gate bf16][up bf16][x][gate codes][up codes]
  static constexpr int kStageBytes = 2 * kABytes + kXBytes + 2 * kRawBytes;  // 40 KB
  static constexpr int kStages = 5;
  static constexpr int kSlabBytes = 32 * kBM * 2;      // 32 tokens x 128 features
  static constexpr int kStagingBytes = 2 * kSlabBytes;
  // Sixteen converter warps (warps 8-23), eight per weight tile: each stage
  // carries two code tiles, so conversion is what bounds this kernel.
  static constexpr int kConvWarps = 16;
  static constexpr int kThreads = (kConvWarp0 + kConvWarps) * kWarp;  // 768
  static constexpr int kTmemCols = 512;                // g: 0-255, u: 256-511
  static constexpr size_t kSmemBytes =
      1024 + static_cast<size_t>(kStages) * kStageBytes + kStagingBytes + 256;
  static_assert(kStageBytes % 1024 == 0, "stage alignment");
};

struct SwigluParams {
  int M, N;
  int num_kb;               // k-blocks of 32
  int kb_per_row;           // scales per weight row (K / 64)
  const float *g_scales;
  const float *u_scales;
  int n_tiles_w;
  int n_tiles_t;            // 256-token blocks; tiles run token-fastest over all of them
  int n_tiles;
  unsigned *err;
};

template <bool kBf16>
__global__ void __launch_bounds__(SwigluCfg::kThreads, 1)
    w8_swiglu_kernel(const __grid_constant__ CUtensorMap tm_x,
                     const __grid_constant__ CUtensorMap tm_g,
                     const __grid_constant__ CUtensorMap tm_u,
                     const __grid_constant__ CUtensorMap tm_y, const SwigluParams p) {
  using C = SwigluCfg;
  constexpr int BT = C::BT;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t *staging = smem + C::kStages * C::kStageBytes;
  uint64_t *bars = reinterpret_cast<uint64_t *>(staging + C::kStagingBytes);
  uint64_t *full = bars;
  uint64_t *empty = bars + C::kStages;
  uint64_t *conv_full = bars + 2 * C::kStages;
  uint64_t *tmem_full = bars + 3 * C::kStages;
  uint64_t *tmem_empty = tmem_full + 1;
  uint64_t *drain = tmem_empty + 1;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
  int *abort_flag = reinterpret_cast<int *>(tmem_slot + 1);

  const int warp = threadIdx.x / kWarp;
  const int lane = threadIdx.x % kWarp;

  if (threadIdx.x == 0) {
    ptx::prefetch_tensor_map(&tm_x);
    ptx::prefetch_tensor_map(&tm_g);
    ptx::prefetch_tensor_map(&tm_u);
    ptx::prefetch_tensor_map(&tm_y);
    for (int s = 0; s < C::kStages; ++s) {
      ptx::mbar_init(&full[s], 1);
      ptx::mbar_init(&empty[s], 1);
      ptx::mbar_init(&conv_full[s], C::kConvWarps);
    }
    ptx::mbar_init(tmem_full, 1);
    ptx::mbar_init(tmem_empty, 4);
    ptx::mbar_init(drain, 1);
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == 1) {
    ptx::tmem_alloc(tmem_slot, C::kTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t outstanding = 0, issue_parity = 0;
      for (int tile = blockIdx.x; tile < p.n_tiles && !aborted(abort_flag); tile += gridDim.x) {
        int tb, fb;
        band_order(tile, p.n_tiles_t, p.n_tiles_w, p.n_tiles_t, tb, fb);
        const int w0 = fb * kBM;
        const int t0 = tb * BT;
        for (int it = 0; it < p.num_kb; ++it) {
          if (!ptx::mbar_wait(&empty[stage], phase ^ 1)) {
            record_timeout(p.err, abort_flag);
            break;
          }
          uint8_t *sx = smem + stage * C::kStageBytes + 2 * C::kABytes;
          uint8_t *raw = sx + C::kXBytes;
          const int k0 = it * C::kBKw;
          ptx::mbar_expect_tx(&full[stage], C::kXBytes + 2 * C::kRawBytes);
          ptx::tma_load_2d(sx, &tm_x, &full[stage], k0, t0);
          ptx::tma_load_2d(raw, &tm_g, &full[stage], k0, w0);
          ptx::tma_load_2d(raw + C::kRawBytes, &tm_u, &full[stage], k0, w0);
          outstanding |= 1u << stage;
          issue_parity = (issue_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (aborted(abort_flag)) {
        for (int s = 0; s < C::kStages; ++s) {
          if (outstanding & (1u << s)) ptx::mbar_wait(&full[s], (issue_parity >> s) & 1u, 200000000ull);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = ptx::make_idesc_f16(kBf16, kBM, BT, false, false);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      for (int tile = blockIdx.x; tile < p.n_tiles && !aborted(abort_flag);
           tile += gridDim.x, ++local) {
        if (!ptx::mbar_wait(tmem_empty, static_cast<uint32_t>(local & 1) ^ 1u)) {
          record_timeout(p.err, abort_flag);
          break;
        }
        ptx::tc_fence_after();
        bool ok = true;
        for (int it = 0; it < p.num_kb; ++it) {
          if (!ptx::mbar_wait(&conv_full[stage], phase)) {
            record_timeout(p.err, abort_flag);
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          const uint32_t sg = ptx::smem_addr(smem + stage * C::kStageBytes);
          const uint32_t su = sg + C::kABytes;
          const uint32_t sx = sg + 2 * C::kABytes;
          for (int ks = 0; ks < C::kBKw / kUmmaK; ++ks) {
            const uint64_t bdesc = kmajor_desc(sx, C::kRowBytes, ks);
            const uint32_t acc = (it > 0 || ks > 0) ? 1u : 0u;
            ptx::mma_f16(tmem_base, kmajor_desc(sg, C::kRowBytes, ks), bdesc, idesc, acc);
            ptx::mma_f16(tmem_base + BT, kmajor_desc(su, C::kRowBytes, ks), bdesc, idesc, acc);
          }
          ptx::mma_commit(&empty[stage]);
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        ptx::mma_commit(tmem_full);
      }
      if (aborted(abort_flag)) {
        ptx::mma_commit(drain);
        ptx::mbar_wait(drain, 0, 200000000ull);
      }
    }
  } else if (warp >= kEpiWarp0 && warp < kEpiWarp0 + 4) {
    // ------------------------------------------------------------------ epilogue
    const int quarter = warp % 4;
    const int row = quarter * 32 + lane;
    const bool elected = threadIdx.x == kEpiWarp0 * kWarp;
    uint32_t slab = 0;
    int local = 0;
    for (int tile = blockIdx.x; tile < p.n_tiles; tile += gridDim.x, ++local) {
      int tb, fb;
      band_order(tile, p.n_tiles_t, p.n_tiles_w, p.n_tiles_t, tb, fb);
      const int w0 = fb * kBM;
      const int t0 = tb * BT;
      // The four epilogue warps share named barriers, so they leave together.
      const bool got = ptx::warp_wait(tmem_full, static_cast<uint32_t>(local & 1));
      if (!ptx::named_bar_all(1, 4 * kWarp, got)) {
        if (lane == 0) record_timeout(p.err, abort_flag);
        break;
      }
      ptx::tc_fence_after();
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
#pragma unroll 1
      for (int c = 0; c < BT / 32; ++c) {
        // Stage a 32-token x 128-feature slab (token-major) and let the TMA
        // engine store it; the slab buffer is double-buffered against the
        // store still reading it.
        if (elected) ptx::bulk_wait_read<1>();
        ptx::named_bar_sync(1, 4 * kWarp);
        uint16_t *stg = reinterpret_cast<uint16_t *>(staging + (slab & 1) * C::kSlabBytes);
#pragma unroll 1
        for (int hh = 0; hh < 2; ++hh) {  // 16 tokens at a time keeps registers low
        uint32_t g[32], u[32];
        ptx::tmem_ld_32x32b_x16(t_row + c * 32 + hh * 16, g);
        ptx::tmem_ld_32x32b_x16(t_row + BT + c * 32 + hh * 16, u);
        ptx::tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 16; j += 2) {
          // The projections' outputs in the activation dtype ...
          const uint32_t gp = kBf16 ? ptx::pack_bf16x2(__uint_as_float(g[j]), __uint_as_float(g[j + 1]))
                                    : ptx::pack_f16x2(__uint_as_float(g[j]), __uint_as_float(g[j + 1]));
          const uint32_t up = kBf16 ? ptx::pack_bf16x2(__uint_as_float(u[j]), __uint_as_float(u[j + 1]))
                                    : ptx::pack_f16x2(__uint_as_float(u[j]), __uint_as_float(u[j + 1]));
          float g0, g1, u0, u1;
          if constexpr (kBf16) {
            g0 = __uint_as_float(gp << 16);
            g1 = __uint_as_float(gp & 0xffff0000u);
            u0 = __uint_as_float(up << 16);
            u1 = __uint_as_float(up & 0xffff0000u);
          } else {
            const float2 gf = __half22float2(*reinterpret_cast<const __half2 *>(&gp));
            const float2 uf = __half22float2(*reinterpret_cast<const __half2 *>(&up));
            g0 = gf.x;
            g1 = gf.y;
            u0 = uf.x;
            u1 = uf.y;
          }
          // ... then silu(g) * u in fp32, rounded once.
          const float h0 = g0 / (1.0f + __expf(-g0)) * u0;
          const float h1 = g1 / (1.0f + __expf(-g1)) * u1;
          const uint32_t hp = kBf16 ? ptx::pack_bf16x2(h0, h1) : ptx::pack_f16x2(h0, h1);
          const int t = hh * 16 + j;
          stg[t * kBM + row] = static_cast<uint16_t>(hp & 0xffffu);
          stg[(t + 1) * kBM + row] = static_cast<uint16_t>(hp >> 16);
        }
        }
        ptx::fence_proxy_async_smem();
        ptx::named_bar_sync(1, 4 * kWarp);
        if (elected) {
          ptx::tma_store_2d(&tm_y, stg, w0, t0 + c * 32);
          ptx::bulk_commit();
        }
        ++slab;
      }
      ptx::tc_fence_before();
      ptx::warp_arrive(tmem_empty);
    }
    if (elected) ptx::bulk_wait_all();  // stores finish reading shared memory before exit
  } else if (warp >= kConvWarp0) {
    // ------------------------------------------------------------------ converters
    // Converter warp cw handles weight tile wt = cw / 8 (0 gate, 1 up); its
    // lane l takes row (cw % 8) * 16 + l / 2, 16-code half l % 2 of the
    // 32-code row, and writes 32 bytes of the 64-byte swizzled bf16 row
    // (logical 16-byte chunk c sits at c ^ ((row >> 1) & 3)).
    const int cw = warp - kConvWarp0;
    const int wt = cw / 8;
    const int r = (cw % 8) * 16 + lane / 2;
    const int half = lane & 1;
    int stage = 0;
    uint32_t phase = 0;
    for (int tile = blockIdx.x; tile < p.n_tiles; tile += gridDim.x) {
      int tb, fb;
      band_order(tile, p.n_tiles_t, p.n_tiles_w, p.n_tiles_t, tb, fb);
      const int w0 = fb * kBM;
      const int n = w0 + r;
      const float *srow =
          n < p.N ? (wt == 0 ? p.g_scales : p.u_scales) + static_cast<int64_t>(n) * p.kb_per_row
                  : nullptr;
      bool ok = true;
      for (int it = 0; it < p.num_kb; ++it) {
        const float sc = srow != nullptr ? __ldg(srow + it / 2) : 0.0f;
        const bool got = ptx::mbar_wait(&full[stage], phase);
        if (__any_sync(0xffffffffu, !got)) {
          if (lane == 0) record_timeout(p.err, abort_flag);
          ok = false;
          break;
        }
        uint8_t *base = smem + stage * C::kStageBytes;
        const uint8_t *raw = base + 2 * C::kABytes + C::kXBytes;
        {
          const int w = wt;
          const uint4 codes =
              *reinterpret_cast<const uint4 *>(raw + w * C::kRawBytes + r * C::kBKw + half * 16);
          const uint32_t words[4] = {codes.x, codes.y, codes.z, codes.w};
          const uint64_t sc2 = ptx::splat_f32x2(sc);
          uint32_t outw[8];
#pragma unroll
          for (int wd = 0; wd < 4; ++wd) {
            const uint32_t uu = words[wd] ^ 0x80808080u;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const uint32_t b0 = __byte_perm(uu, 0x4B000000u, 0x7440u | (2 * h));
              const uint32_t b1 = __byte_perm(uu, 0x4B000000u, 0x7440u | (2 * h + 1));
              float lo, hi;
              ptx::dequant_pair(b0, b1, sc2, lo, hi);
              outw[2 * wd + h] = kBf16 ? ptx::pack_bf16x2(lo, hi) : ptx::pack_f16x2(lo, hi);
            }
          }
          uint8_t *dst_row = base + w * C::kABytes + r * C::kRowBytes;
          const int sw = (r >> 1) & 3;
          *reinterpret_cast<uint4 *>(dst_row + (((2 * half) ^ sw) << 4)) =
              make_uint4(outw[0], outw[1], outw[2], outw[3]);
          *reinterpret_cast<uint4 *>(dst_row + (((2 * half + 1) ^ sw) << 4)) =
              make_uint4(outw[4], outw[5], outw[6], outw[7]);
        }
        ptx::fence_proxy_async_smem();
        ptx::warp_arrive(&conv_full[stage]);
        if (++stage == C::kStages) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (!ok) break;
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem_base, C::kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// Host side: tensor maps and launches.
// ---------------------------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                   const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                   const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static std::atomic<EncodeTiledFn> cached{nullptr};
  EncodeTiledFn fn = cached.load(std::memory_order_acquire);
  if (fn != nullptr) return fn;
  void *sym = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &sym, cudaEnableDefault, &q) !=
          cudaSuccess ||
      q != cudaDriverEntryPointSuccess || sym == nullptr) {
    return nullptr;
  }
  fn = reinterpret_cast<EncodeTiledFn>(sym);
  cached.store(fn, std::memory_order_release);
  return fn;
}

// Launch attribute of the linear kernels: they may begin while the
// down-projection launched just before them on the stream is still running
// (their producers wait for it before reading P).
void set_programmatic_dependency(cudaLaunchAttribute &attr) {
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
}

CUtensorMapSwizzle swizzle_for(int inner_bytes) {
  switch (inner_bytes) {
    case 32: return CU_TENSOR_MAP_SWIZZLE_32B;
    case 64: return CU_TENSOR_MAP_SWIZZLE_64B;
    case 128: return CU_TENSOR_MAP_SWIZZLE_128B;
    default: return CU_TENSOR_MAP_SWIZZLE_NONE;
  }
}

// 2-D row-major tensor [outer, inner] with element size esize, box [box_outer, box_inner].
int make_map(CUtensorMap *map, const void *base, int esize, int64_t inner, int64_t outer,
             int box_inner, int box_outer, bool swizzle) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return record_cuda_error(cudaErrorNotSupported);
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(inner) * esize};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(box_inner), static_cast<cuuint32_t>(box_outer)};
  const cuuint32_t estr[2] = {1, 1};
  const CUtensorMapDataType dt = esize == 1   ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                 : esize == 2 ? CU_TENSOR_MAP_DATA_TYPE_UINT16
                                              : CU_TENSOR_MAP_DATA_TYPE_UINT32;
  const CUresult r = fn(map, dt, 2, const_cast<void *>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle ? swizzle_for(box_inner * esize) : CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? CF_OK : CF_ERR_UNSUPPORTED;
}

template <int BN, bool kBf16>
int launch_gemm(const CUtensorMap &a, const CUtensorMap &b, const CUtensorMap &pa,
                const CUtensorMap &pb, const GemmParams &params, cudaStream_t stream) {
  using C = GemmCfg<BN>;
  auto kernel = lora_gemm_kernel<BN, kBf16>;
  if (int st = allow_dynamic_smem<lora_gemm_kernel<BN, kBf16>>(C::kSmemBytes)) return st;
  const int grid = std::max(1, std::min(params.n_tiles, sm_count()));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(C::kThreads);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  set_programmatic_dependency(attr[0]);
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  CFB_TRY_CUDA(cudaLaunchKernelEx(&cfg, kernel, a, b, pa, pb, params));
  return check_launch();
}

// Down-projection workspace P [m, r]: 16-bit for bf16/f16 calls, fp32 for
// fp32 calls.
size_t workspace_bytes(int64_t m, int64_t r, int elem_bytes = 2) {
  if (m <= 0 || r <= 0) return 0;
  const size_t bytes = static_cast<size_t>(m) * static_cast<size_t>(r) * elem_bytes;
  return (bytes + 255) & ~static_cast<size_t>(255);
}

struct LinearArgs {
  const void *x;
  const void *w;          // bf16/f16 weight, or int8 codes
  int w_layout;           // CF_LAYOUT_REF ([K, N]) or CF_LAYOUT_T ([N, K]); int8: [N, K]
  const float *w_scales;  // int8 only
  const void *a;
  int a_layout;
  const void *b;
  int b_layout;
  void *y;
  int64_t m, k, n, r;
  float scale;
  int dtype;
  void *ws;
  size_t ws_bytes;
  bool int8;
  // Fused all-gather (W8 only): every destination receives this call's
  // features at columns [col0, col0 + n) of a [m, ldy] matrix.
  int n_dest = 0;
  void *const *dest = nullptr;
  int64_t ldy = 0;
  int64_t col0 = 0;
  int self_dest = 0;  // index in dest of this GPU's own copy
  void *mc = nullptr;  // multicast address of the destination (multimem epilogue)
  // Folded RMSNorm (wide kernel only): x is the un-normalised residual sum.
  const void *norm_w = nullptr;  // fp32 [K]
  const float *row_scale = nullptr;
  // Row-group completion counters for a copy-engine all-gather (wide kernel).
  unsigned *done = nullptr;
  int rb_per_group = 1;
  int n_groups = 0;
};

template <int R, bool kBf16>
int launch_down_projection(const LinearArgs &L, unsigned *err, cudaStream_t stream) {
  using C = DownCfg<R>;
  CUtensorMap tm_x, tm_a;
  if (int st = make_map(&tm_x, L.x, 2, L.k, L.m, kBK, kBM, true)) return st;
  DownParams p{};
  p.M = static_cast<int>(L.m);
  p.num_kb = static_cast<int>((L.k + kBK - 1) / kBK);
  p.scale = L.scale;
  p.out = L.ws;
  p.err = err;
  if (L.a_layout == CF_LAYOUT_REF) {
    // a [K, r]: r contiguous -> MN-major B operand, one swizzle row of r elements.
    if (int st = make_map(&tm_a, L.a, 2, R, L.k, R, kBK, true)) return st;
    p.a_mn_major = 1;
  } else {
    // a^T [r, K]: K contiguous -> K-major B operand.
    if (int st = make_map(&tm_a, L.a, 2, L.k, R, kBK, R, true)) return st;
    p.a_mn_major = 0;
  }
  // Split K over up to 8 CTAs per row tile while the grid stays within one wave.
  const int m_tiles = static_cast<int>((L.m + kBM - 1) / kBM);
  int splits = 1;
  while (splits < 8 && m_tiles * splits * 2 <= sm_count() && splits * 2 <= p.num_kb) splits *= 2;
  p.splits = splits;
  p.kb_per_split = (p.num_kb + splits - 1) / splits;

  auto kernel = down_proj_kernel<R, kBf16>;
  if (int st_ = allow_dynamic_smem<down_proj_kernel<R, kBf16>>(C::kSmemBytes)) return st_;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(m_tiles * splits));
  cfg.blockDim = dim3(C::kThreads);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(splits);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  CFB_TRY_CUDA(cudaLaunchKernelEx(&cfg, kernel, tm_x, tm_a, p));
  return check_launch();
}

template <int BT, bool kBf16>
int launch_w8_decode(const LinearArgs &L, unsigned *err, cudaStream_t stream) {
  using C = DecCfg<BT>;
  const int r = static_cast<int>(L.r);
  CUtensorMap tm_x, tm_codes, tm_p, tm_bt;
  int st = CF_OK;
  if ((st = make_map(&tm_x, L.x, 2, L.k, L.m, kBK, BT, true))) return st;
  // 128-byte swizzled code rows: a converter warp's eight rows then read
  // eight different bank groups instead of the same one.
  if ((st = make_map(&tm_codes, L.w, 1, L.k, L.n, kBK * C::kRawKb, kBM, true))) return st;
  if ((st = make_map(&tm_p, L.ws, 2, r, L.m, r, BT, true))) return st;
  DecParams p{};
  if (L.b_layout == CF_LAYOUT_REF) {
    // b [r, N]: N contiguous -> MN-major A operand, chunks of 64 features x r.
    if ((st = make_map(&tm_bt, L.b, 2, L.n, r, 64, r, true))) return st;
    p.b_mn = 1;
  } else {
    // b^T [N, r]: r contiguous -> K-major A operand.
    if ((st = make_map(&tm_bt, L.b, 2, r, L.n, r, kBM, true))) return st;
    p.b_mn = 0;
  }
  p.M = static_cast<int>(L.m);
  p.N = static_cast<int>(L.n);
  p.num_kb = static_cast<int>(L.k / kBK);
  p.rank = r;
  p.w_scales = L.w_scales;
  p.out = static_cast<uint16_t *>(L.y);
  p.err = err;
  CUtensorMap tm_scales;
  std::memset(&tm_scales, 0, sizeof(tm_scales));
  // scales as an fp32 [N, num_kb] matrix in boxes of 4 x 128: needs 16-byte rows
  p.scale_tma = (p.num_kb % 4 == 0 && aligned_to(L.w_scales, 16)) ? 1 : 0;
  if (p.scale_tma) {
    if ((st = make_map(&tm_scales, L.w_scales, 4, p.num_kb, L.n, 4, kBM, false))) return st;
  }
  const int n_tiles = static_cast<int>((L.n + kBM - 1) / kBM);
  // Largest K split (cluster size <= 8) that keeps the whole grid resident.
  const int slots = sm_count() * C::kMinBlocks;
  int splits = 1;
  for (int s = 8; s >= 2; --s) {
    if (n_tiles * s <= slots && s <= p.num_kb) {
      splits = s;
      break;
    }
  }
  p.splits = splits;
  // Whole raw stages per CTA: every slice but the last starts on a stage.
  p.kb_per_split = ((p.num_kb + splits - 1) / splits + C::kRawKb - 1) / C::kRawKb * C::kRawKb;
  auto kernel = w8_decode_kernel<BT, kBf16>;
  if (int st_ = allow_dynamic_smem<w8_decode_kernel<BT, kBf16>>(C::kSmemBytes)) return st_;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(n_tiles * splits));
  cfg.blockDim = dim3(C::kThreads);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(splits);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  set_programmatic_dependency(attr[1]);
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  CFB_TRY_CUDA(cudaLaunchKernelEx(&cfg, kernel, tm_x, tm_codes, tm_p, tm_bt, tm_scales, p));
  return check_launch();
}

template <bool kBf16, bool kTmaStore, int kBT, bool kNorm = false>
int launch_w8_wide(const LinearArgs &L, unsigned *err, cudaStream_t stream) {
  using C = W8WideCfg<kTmaStore, kBT>;
  const int r = static_cast<int>(L.r);
  CUtensorMap tm_x, tm_codes, tm_p, tm_bt;
  int st = CF_OK;
  if ((st = make_map(&tm_x, L.x, 2, L.k, L.m, C::kBKw, 256, true))) return st;
  if ((st = make_map(&tm_codes, L.w, 1, L.k, L.n, C::kBKw, kBM, false))) return st;
  if ((st = make_map(&tm_p, L.ws, 2, r, L.m, kUmmaK, 256, true))) return st;
  W8Params p{};
  if (L.b_layout == CF_LAYOUT_REF) {
    if ((st = make_map(&tm_bt, L.b, 2, L.n, r, 64, kUmmaK, true))) return st;
    p.extra_b_mn = 1;
  } else {
    if ((st = make_map(&tm_bt, L.b, 2, r, L.n, kUmmaK, kBM, true))) return st;
    p.extra_b_mn = 0;
  }
  p.M = static_cast<int>(L.m);
  p.N = static_cast<int>(L.n);
  p.num_kb = static_cast<int>(L.k / C::kBKw);
  p.extra_ksteps = r / kUmmaK;
  p.rank = r;
  p.w_scales = L.w_scales;
  p.kb_per_row = static_cast<int>(L.k / kBK);
  CUtensorMap tm_scales;
  std::memset(&tm_scales, 0, sizeof(tm_scales));
  p.scale_tma = (p.kb_per_row % 4 == 0 && aligned_to(L.w_scales, 16)) ? 1 : 0;
  if (p.scale_tma) {
    if ((st = make_map(&tm_scales, L.w_scales, 4, p.kb_per_row, L.n, 4, kBM, false))) return st;
  }
  OutMaps out_maps;
  std::memset(&out_maps, 0, sizeof(out_maps));
  if (L.n_dest > 0) {
    p.ldo = static_cast<int>(L.ldy);
    p.out_col0 = static_cast<int>(L.col0);
    p.n_outs = L.n_dest;
    p.self_out = L.self_dest;
    for (int d = 0; d < L.n_dest; ++d) p.outs[d] = L.dest[d];
  } else {
    p.ldo = static_cast<int>(L.n);
    p.out_col0 = 0;
    p.n_outs = 1;
    p.outs[0] = L.y;
  }
  if (kTmaStore) {
    for (int d = 0; d < p.n_outs; ++d) {
      if ((st = make_map(&out_maps.map[d], p.outs[d], 2, p.ldo, L.m, kBM, 32, false))) return st;
    }
  }
  p.n_tiles_w = static_cast<int>((L.n + kBM - 1) / kBM);
  p.n_tiles = p.n_tiles_w * static_cast<int>((L.m + C::BT - 1) / C::BT);
  p.err = err;
  p.done = kTmaStore ? L.done : nullptr;
  p.mc_out = kTmaStore ? L.mc : nullptr;
  p.rb_per_group = L.rb_per_group;
  p.n_groups = L.n_groups;
  p.norm_w = static_cast<const float *>(L.norm_w);
  CUtensorMap tm_norm;
  std::memset(&tm_norm, 0, sizeof(tm_norm));
  if (kNorm) {
    if ((st = make_map(&tm_norm, L.norm_w, 4, L.k, 1, C::kBKw, 1, false))) return st;
  }
  p.row_scale = L.row_scale;
  auto kernel = w8_wide_kernel<kBf16, kTmaStore, kBT, kNorm>;
  if (int st_ = allow_dynamic_smem<w8_wide_kernel<kBf16, kTmaStore, kBT, kNorm>>(C::kSmemBytes)) {
    return st_;
  }
  const int grid = std::max(1, std::min(p.n_tiles, sm_count()));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(C::kThreads);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  set_programmatic_dependency(attr[0]);
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  CFB_TRY_CUDA(cudaLaunchKernelEx(&cfg, kernel, tm_x, tm_codes, tm_p, tm_bt, tm_scales, tm_norm,
                                  out_maps, p));
  return check_launch();
}

template <bool kBf16>
int run_linear(const LinearArgs &L, cudaStream_t stream) {
  unsigned *err = device_error_word();
  if (err == nullptr) return record_cuda_error(cudaGetLastError());
  int st = CF_OK;
  switch (L.r) {
    case 16: st = launch_down_projection<16, kBf16>(L, err, stream); break;
    case 32: st = launch_down_projection<32, kBf16>(L, err, stream); break;
    default: st = launch_down_projection<64, kBf16>(L, err, stream); break;
  }
  if (st != CF_OK) return st;
  if (L.int8) {
    if (L.norm_w != nullptr) return launch_w8_wide<kBf16, true, 512, true>(L, err, stream);
    if (L.n_dest == 0 && L.m <= 32) return launch_w8_decode<32, kBf16>(L, err, stream);
    if (L.n_dest == 0 && L.m <= 64) return launch_w8_decode<64, kBf16>(L, err, stream);
    if (L.n_dest == 0 && L.m <= 128) return launch_w8_decode<128, kBf16>(L, err, stream);
    // Every call runs 512-token tiles (the 256-token, two-accumulator form
    // kept for measurement overlapped the multicast stores at 8 GPUs, 1.81
    // against 1.86 ms, but was 35 % slower at 2 GPUs and on one GPU).
    return launch_w8_wide<kBf16, true, 512>(L, err, stream);
  }

  constexpr int BN = 256;
  const int r = static_cast<int>(L.r);
  CUtensorMap tm_x, tm_w, tm_p, tm_b;
  if ((st = make_map(&tm_x, L.x, 2, L.k, L.m, kBK, kBM, true))) return st;
  GemmParams p{};
  if (L.w_layout == CF_LAYOUT_T) {
    if ((st = make_map(&tm_w, L.w, 2, L.k, L.n, kBK, BN, true))) return st;
    p.b_src = kBKMajor;
  } else {
    if ((st = make_map(&tm_w, L.w, 2, L.n, L.k, 64, kBK, true))) return st;
    p.b_src = kBMNMajor;
  }
  if ((st = make_map(&tm_p, L.ws, 2, r, L.m, r, kBM, true))) return st;
  if (L.b_layout == CF_LAYOUT_REF) {
    // b [r, N]: N contiguous -> MN-major, chunks of 64 columns x r rows.
    if ((st = make_map(&tm_b, L.b, 2, L.n, r, 64, r, true))) return st;
    p.extra_b_mn = 1;
  } else {
    // b^T [N, r]: r contiguous -> K-major rows of r elements.
    if ((st = make_map(&tm_b, L.b, 2, r, L.n, r, BN, true))) return st;
    p.extra_b_mn = 0;
  }
  p.M = static_cast<int>(L.m);
  p.N = static_cast<int>(L.n);
  p.K = static_cast<int>(L.k);
  p.num_kb = static_cast<int>((L.k + kBK - 1) / kBK);
  p.extra_ksteps = r / kUmmaK;
  p.rank = r;
  p.is_bf16 = kBf16;
  p.out_scale = 1.0f;
  p.out = L.y;
  p.ldo = static_cast<int>(L.n);
  p.n_tiles_n = static_cast<int>((L.n + BN - 1) / BN);
  p.n_tiles = static_cast<int>((L.m + kBM - 1) / kBM) * p.n_tiles_n;
  p.err = err;
  return launch_gemm<BN, kBf16>(tm_x, tm_w, tm_p, tm_b, p, stream);
}

// Row blocks per band of the fp32 kernel's tile walk: as many 128-row blocks
// of the [m, k] fp32 A operand as fit in 32 MB, so a band stays in L2 while
// the B column blocks stream past it.
int f32_band(int m_tiles, int64_t k) {
  const int64_t block_bytes = 128 * std::max<int64_t>(k, 1) * 4;
  const int64_t fit = (int64_t{32} << 20) / block_bytes;
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(m_tiles, fit)));
}

// fp32 call: two launches of lora_f32_kernel (down-projection, then the main
// product with the adapter as extra k-blocks), the second overlapping the
// first through programmatic dependent launch.
int launch_f32(const CUtensorMap &a, const CUtensorMap &b, const CUtensorMap &pa,
               const CUtensorMap &pb, const F32Params &p, bool dependent, cudaStream_t stream) {
  if (int st = allow_dynamic_smem<lora_f32_kernel>(F32Cfg::kSmemBytes)) return st;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(std::max(1, std::min(p.n_tiles, sm_count()))));
  cfg.blockDim = dim3(F32Cfg::kThreads);
  cfg.dynamicSmemBytes = F32Cfg::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  set_programmatic_dependency(attr[0]);
  cfg.attrs = attr;
  cfg.numAttrs = dependent ? 1 : 0;
  CFB_TRY_CUDA(cudaLaunchKernelEx(&cfg, lora_f32_kernel, a, b, pa, pb, p));
  return check_launch();
}

// Map of an fp32 B operand: [K, N] (N contiguous) as 32-column x 32-row
// MN-major chunks, or [N, K] as 128 rows of 32 K-major elements.
int make_f32_b_map(CUtensorMap *map, const void *base, bool mn, int64_t k, int64_t n) {
  return mn ? make_map(map, base, 4, n, k, 32, 32, true) : make_map(map, base, 4, k, n, 32, 128, true);
}

int run_linear_f32(const LinearArgs &L, cudaStream_t stream) {
  unsigned *err = device_error_word();
  if (err == nullptr) return record_cuda_error(cudaGetLastError());
  const int r = static_cast<int>(L.r);
  const bool a_mn = L.a_layout == CF_LAYOUT_REF;  // A [K, r]: r contiguous
  const bool w_mn = L.w_layout == CF_LAYOUT_REF;  // W [K, N]: N contiguous
  const bool b_mn = L.b_layout == CF_LAYOUT_REF;  // B [r, N]: N contiguous
  CUtensorMap tm_x, tm_a, tm_w, tm_p, tm_b;
  int st = CF_OK;
  if ((st = make_map(&tm_x, L.x, 4, L.k, L.m, 32, 128, true))) return st;
  if ((st = make_f32_b_map(&tm_a, L.a, a_mn, L.k, r))) return st;
  if ((st = make_f32_b_map(&tm_w, L.w, w_mn, L.k, L.n))) return st;
  if ((st = make_map(&tm_p, L.ws, 4, r, L.m, 32, 128, true))) return st;
  if ((st = make_f32_b_map(&tm_b, L.b, b_mn, r, L.n))) return st;
  const int m_tiles = static_cast<int>((L.m + 127) / 128);
  F32Params d{};
  d.M = static_cast<int>(L.m);
  d.N = r;
  d.num_kb = static_cast<int>((L.k + F32Cfg::kBKf - 1) / F32Cfg::kBKf);
  d.extra_kb = 0;
  d.n_mma = r;
  d.b_mn = a_mn ? 1 : 0;
  d.e_mn = 0;
  d.ldo = r;
  d.products = 3;
  d.out_scale = L.scale;
  d.out = static_cast<float *>(L.ws);
  d.n_tiles_n = 1;
  d.n_tiles_m = m_tiles;
  d.band_m = m_tiles;
  d.n_tiles = m_tiles;
  d.err = err;
  if ((st = launch_f32(tm_x, tm_a, tm_x, tm_a, d, false, stream))) return st;
  F32Params p = d;
  p.N = static_cast<int>(L.n);
  p.extra_kb = (r + F32Cfg::kBKf - 1) / F32Cfg::kBKf;
  p.n_mma = F32Cfg::BN;
  p.b_mn = w_mn ? 1 : 0;
  p.e_mn = b_mn ? 1 : 0;
  p.ldo = static_cast<int>(L.n);
  p.out_scale = 1.0f;
  p.out = static_cast<float *>(L.y);
  p.n_tiles_n = static_cast<int>((L.n + F32Cfg::BN - 1) / F32Cfg::BN);
  p.band_m = f32_band(m_tiles, L.k);
  p.n_tiles = m_tiles * p.n_tiles_n;
  return launch_f32(tm_x, tm_w, tm_p, tm_b, p, true, stream);
}

// c [m, n] = a [m, k] b [k, n] in fp32 (one launch of lora_f32_kernel with
// no adapter).
int run_matmul_f32(const float *a, const float *b, int b_layout, float *c, int64_t m, int64_t n,
                   int64_t k, int precise, cudaStream_t stream) {
  unsigned *err = device_error_word();
  if (err == nullptr) return record_cuda_error(cudaGetLastError());
  const bool b_mn = b_layout == CF_LAYOUT_REF;
  CUtensorMap tm_a, tm_b;
  int st = CF_OK;
  if ((st = make_map(&tm_a, a, 4, k, m, 32, 128, true))) return st;
  if ((st = make_f32_b_map(&tm_b, b, b_mn, k, n))) return st;
  F32Params p{};
  p.M = static_cast<int>(m);
  p.N = static_cast<int>(n);
  p.num_kb = static_cast<int>((k + F32Cfg::kBKf - 1) / F32Cfg::kBKf);
  p.extra_kb = 0;
  p.n_mma = F32Cfg::BN;
  p.b_mn = b_mn ? 1 : 0;
  p.ldo = static_cast<int>(n);
  p.products = precise ? 3 : 1;
  p.out_scale = 1.0f;
  p.out = c;
  p.n_tiles_n = static_cast<int>((n + F32Cfg::BN - 1) / F32Cfg::BN);
  p.n_tiles_m = static_cast<int>((m + 127) / 128);
  p.band_m = f32_band(p.n_tiles_m, k);
  p.n_tiles = p.n_tiles_m * p.n_tiles_n;
  p.err = err;
  return launch_f32(tm_a, tm_b, tm_a, tm_b, p, false, stream);
}

template <bool kBf16>
int run_merge_quantize(const void *w, const void *lora_a, const void *lora_b, int64_t n,
                       int64_t k, int64_t r, float scaling, int8_t *codes, float *scales,
                       cudaStream_t stream) {
  unsigned *err = device_error_word();
  if (err == nullptr) return record_cuda_error(cudaGetLastError());
  CUtensorMap tm_b, tm_a;
  int st = CF_OK;
  // lora_b [n, r]: K-major rows of r elements; lora_a [r, k]: 64-column chunks;
  // W [n, k]: 64-column boxes of 128 rows.
  CUtensorMap tm_w;
  if ((st = make_map(&tm_b, lora_b, 2, r, n, r, kBM, true))) return st;
  if ((st = make_map(&tm_a, lora_a, 2, k, r, 64, r, true))) return st;
  if ((st = make_map(&tm_w, w, 2, k, n, 64, kBM, true))) return st;
  MergeParams p{};
  p.N = static_cast<int>(n);
  p.K = static_cast<int>(k);
  p.rank = static_cast<int>(r);
  p.scaling = scaling;
  p.w = static_cast<const uint16_t *>(w);
  p.codes = codes;
  p.scales = scales;
  p.n_tiles_k = static_cast<int>((k + MergeCfg::BK - 1) / MergeCfg::BK);
  p.n_tiles = p.n_tiles_k * static_cast<int>((n + kBM - 1) / kBM);
  p.err = err;
  if ((st = allow_dynamic_smem<lora_merge_quant_kernel<kBf16>>(MergeCfg::kSmemBytes))) return st;
  const int grid = std::max(1, std::min(p.n_tiles, sm_count()));
  lora_merge_quant_kernel<kBf16><<<grid, MergeCfg::kThreads, MergeCfg::kSmemBytes, stream>>>(
      tm_b, tm_a, tm_w, p);
  return check_launch();
}

template <bool kBf16>
int run_w8_swiglu(const void *x, const int8_t *g_codes, const float *g_scales,
                  const int8_t *u_codes, const float *u_scales, void *y, int64_t m, int64_t k,
                  int64_t n, cudaStream_t stream) {
  using C = SwigluCfg;
  unsigned *err = device_error_word();
  if (err == nullptr) return record_cuda_error(cudaGetLastError());
  CUtensorMap tm_x, tm_g, tm_u, tm_y;
  int st = CF_OK;
  if ((st = make_map(&tm_x, x, 2, k, m, C::kBKw, C::BT, true))) return st;
  if ((st = make_map(&tm_g, g_codes, 1, k, n, C::kBKw, kBM, false))) return st;
  if ((st = make_map(&tm_u, u_codes, 1, k, n, C::kBKw, kBM, false))) return st;
  if ((st = make_map(&tm_y, y, 2, n, m, kBM, 32, false))) return st;
  SwigluParams p{};
  p.M = static_cast<int>(m);
  p.N = static_cast<int>(n);
  p.num_kb = static_cast<int>(k / C::kBKw);
  p.kb_per_row = static_cast<int>(k / kQuantBlockSize);
  p.g_scales = g_scales;
  p.u_scales = u_scales;
  p.n_tiles_w = static_cast<int>((n + kBM - 1) / kBM);
  p.n_tiles_t = static_cast<int>((m + C::BT - 1) / C::BT);
  p.n_tiles = p.n_tiles_w * p.n_tiles_t;
  p.err = err;
  if ((st = allow_dynamic_smem<w8_swiglu_kernel<kBf16>>(C::kSmemBytes))) return st;
  const int grid = std::max(1, std::min(p.n_tiles, sm_count()));
  w8_swiglu_kernel<kBf16><<<grid, C::kThreads, C::kSmemBytes, stream>>>(tm_x, tm_g, tm_u, tm_y, p);
  return check_launch();
}

int validate_and_run(const LinearArgs &L, cf_stream_t stream) {
  if (L.m < 0 || L.k < 0 || L.n < 0 || L.r < 0) return CF_ERR_INVALID_ARGUMENT;
  if (L.m == 0 || L.n == 0) return CF_OK;
  if (L.x == nullptr || L.w == nullptr || L.a == nullptr || L.b == nullptr || L.y == nullptr ||
      (L.int8 && L.w_scales == nullptr)) {
    return CF_ERR_INVALID_ARGUMENT;
  }
  const bool f32 = L.dtype == CF_DTYPE_F32;
  if (L.dtype != CF_DTYPE_BF16 && L.dtype != CF_DTYPE_F16 && !(f32 && !L.int8)) {
    return CF_ERR_UNSUPPORTED;
  }
  if (L.r != 16 && L.r != 32 && L.r != 64) return CF_ERR_UNSUPPORTED;
  // Row strides must be whole 16-byte units for TMA.
  const int64_t k_align = L.int8 ? kBK : (f32 ? 4 : 8);
  if (L.k == 0 || L.k % k_align != 0 || L.n % (f32 ? 4 : 8) != 0) return CF_ERR_UNSUPPORTED;
  if ((L.w_layout != CF_LAYOUT_REF && L.w_layout != CF_LAYOUT_T) ||
      (L.a_layout != CF_LAYOUT_REF && L.a_layout != CF_LAYOUT_T) ||
      (L.b_layout != CF_LAYOUT_REF && L.b_layout != CF_LAYOUT_T)) {
    return CF_ERR_INVALID_ARGUMENT;
  }
  if (L.m > INT32_MAX || L.n > INT32_MAX || L.k > INT32_MAX) return CF_ERR_UNSUPPORTED;
  for (const void *ptr : {L.x, L.w, L.a, L.b, static_cast<const void *>(L.y)}) {
    if (!aligned_to(ptr, 16)) return CF_ERR_MISALIGNED;
  }
  if (L.ws == nullptr || L.ws_bytes < workspace_bytes(L.m, L.r, f32 ? 4 : 2)) {
    return CF_ERR_WORKSPACE;
  }
  if (!aligned_to(L.ws, 16)) return CF_ERR_MISALIGNED;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (f32) return run_linear_f32(L, s);
  return L.dtype == CF_DTYPE_BF16 ? run_linear<true>(L, s) : run_linear<false>(L, s);
}

// A'[k, j] = w[k] * A[k, j] in the dtype ([K, r], K-major rows of r): the
// norm weight folded into the down-projection, so P' = scale * h A' needs no
// normalised copy of h. `a` is [K, r] (a_t = 0) or [r, K] (a_t = 1).
template <typename T>
__global__ void weight_adapter_kernel(const T *a, int a_t, const T *w, T *out, float *w32,
                                      int64_t k, int64_t r) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < k;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    w32[i] = static_cast<float>(w[i]);
  }
  const int64_t total = k * r;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t kk = i / r, j = i % r;
    const float v = static_cast<float>(a[a_t ? j * k + kk : i]) * static_cast<float>(w[kk]);
    out[i] = static_cast<T>(v);
  }
}

size_t align256(size_t b) { return (b + 255) & ~static_cast<size_t>(255); }

// Workspace of cf_rmsnorm_lora_linear_int8: the folded route needs the row
// scales, A' and P; the route for short token counts (decode kernel) needs a
// normalised copy of x and P.
size_t norm_linear_workspace(int64_t m, int64_t k, int64_t r) {
  if (m <= 0 || k <= 0 || r <= 0) return 0;
  const size_t p = workspace_bytes(m, r, 2);
  const size_t folded = align256(static_cast<size_t>(m) * 4) + align256(static_cast<size_t>(k) * 4) +
                        align256(static_cast<size_t>(k * r) * 2) + p;
  const size_t plain = align256(static_cast<size_t>(m * k) * 2) + p;
  return std::max(folded, plain);
}

}  // namespace
}  // namespace cfb

// ---------------------------------------------------------------------------
// Allocation-free variant of cf_lora_linear.
//
// Some callers cannot allocate device memory for the down-projection
// workspace: a host whose device memory is reserved up front by another
// allocator (a serving engine that hands all free HBM to its KV cache or its
// own pool), a foreign-language host bound to this C ABI with no CUDA
// allocator of its own, and latency-critical loops that must not pay
// cudaMalloc's implicit device synchronisation per layer. For them the
// workspace lives in this file-scope device array, which every GPU that loads
// the library holds until the process exits.
//
// Limits and rules:
//   * at most kNoAllocScratchBytes (4 MiB) of workspace: m * rank * 2 bytes
//     (4 for fp32 calls), rounded up to 256 (bf16/f16: m <= 131072 at rank 16,
//     m <= 32768 at rank 64);
//     larger calls return CF_ERR_WORKSPACE and launch nothing;
//   * the array is shared by every call on a device and keeps the last call's
//     contents. Nothing needs to start at zero: each call's down-projection
//     overwrites the rows it reads. Calls whose kernels overlap on the GPU
//     (different streams without ordering) race on it;
//   * the first call on a device looks up the array's device address with
//     cudaGetSymbolAddress (once per device, with that device current); make
//     that first call before any stream capture.
// ---------------------------------------------------------------------------
namespace cfb {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t{4} << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::atomic<void *> g_noalloc_ptr[64];

// Device address of g_noalloc_scratch on the current device (set up once per
// device). In host code the array's name is only a host-side stand-in.
int noalloc_scratch(void **out) {
  int dev = 0;
  CFB_TRY_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return CF_ERR_UNSUPPORTED;
  void *ptr = g_noalloc_ptr[dev].load(std::memory_order_acquire);
  if (ptr == nullptr) {
    CFB_TRY_CUDA(cudaGetSymbolAddress(&ptr, g_noalloc_scratch));
    g_noalloc_ptr[dev].store(ptr, std::memory_order_release);
  }
  *out = ptr;
  return CF_OK;
}

}  // namespace
}  // namespace cfb

extern "C" {

int cf_lora_linear_noalloc(const void *x, const void *w, int w_layout, const void *a,
                           int a_layout, const void *b, int b_layout, void *y, int64_t m,
                           int64_t k, int64_t n, int64_t rank, float scale, int dtype,
                           cf_stream_t stream) {
  if (m < 0 || rank < 0) return CF_ERR_INVALID_ARGUMENT;
  const size_t need = cfb::workspace_bytes(m, rank, dtype == CF_DTYPE_F32 ? 4 : 2);
  if (need > cfb::kNoAllocScratchBytes) return CF_ERR_WORKSPACE;
  void *scratch = nullptr;
  if (m > 0 && n > 0) {
    if (int st = cfb::noalloc_scratch(&scratch)) return st;
  }
  cfb::LinearArgs L{x, w, w_layout, nullptr, a, a_layout, b, b_layout, y, m, k, n, rank,
                    scale, dtype, scratch, cfb::kNoAllocScratchBytes, false};
  return cfb::validate_and_run(L, stream);
}

size_t cf_lora_linear_workspace_bytes(int64_t m, int64_t rank) {
  // Enough for every dtype (fp32 calls keep P in fp32).
  return cfb::workspace_bytes(m, rank, 4);
}

int cf_lora_linear(const void *x, const void *w, int w_layout, const void *a, int a_layout,
                   const void *b, int b_layout, void *y, int64_t m, int64_t k, int64_t n,
                   int64_t rank, float scale, int dtype, void *workspace, size_t workspace_bytes,
                   cf_stream_t stream) {
  cfb::LinearArgs L{x, w, w_layout, nullptr, a, a_layout, b, b_layout, y, m, k, n, rank,
                    scale, dtype, workspace, workspace_bytes, false};
  return cfb::validate_and_run(L, stream);
}

int cf_lora_linear_int8(const void *x, const int8_t *w_codes, const float *w_scales,
                        const void *a, int a_layout, const void *b, int b_layout, void *y,
                        int64_t m, int64_t k, int64_t n, int64_t rank, float scale, int dtype,
                        void *workspace, size_t workspace_bytes, cf_stream_t stream) {
  cfb::LinearArgs L{x, w_codes, CF_LAYOUT_T, w_scales, a, a_layout, b, b_layout, y, m, k, n,
                    rank, scale, dtype, workspace, workspace_bytes, true};
  if (w_scales != nullptr && !cfb::aligned_to(w_scales, 4)) return CF_ERR_MISALIGNED;
  return cfb::validate_and_run(L, stream);
}

int cf_lora_linear_int8_allgather(const void *x, const int8_t *w_codes, const float *w_scales,
                                  const void *a, int a_layout, const void *b, int b_layout,
                                  int n_dest, void *const *y_dest, int self_dest, int64_t ldy,
                                  int64_t col0, int64_t m, int64_t k, int64_t n, int64_t rank,
                                  float scale, int dtype, void *workspace, size_t workspace_bytes,
                                  cf_stream_t stream) {
  if (n_dest < 1 || n_dest > cfb::kMaxOuts || y_dest == nullptr) return CF_ERR_INVALID_ARGUMENT;
  if (self_dest < 0 || self_dest >= n_dest) return CF_ERR_INVALID_ARGUMENT;
  for (int d = 0; d < n_dest; ++d) {
    if (y_dest[d] == nullptr) return CF_ERR_INVALID_ARGUMENT;
    if (!cfb::aligned_to(y_dest[d], 16)) return CF_ERR_MISALIGNED;
  }
  if (ldy <= 0 || col0 < 0 || col0 + n > ldy) return CF_ERR_INVALID_ARGUMENT;
  if (ldy % 8 != 0 || col0 % 8 != 0 || ldy > INT32_MAX || n % 128 != 0) return CF_ERR_UNSUPPORTED;
  cfb::LinearArgs L{x, w_codes, CF_LAYOUT_T, w_scales, a, a_layout, b, b_layout,
                    y_dest[self_dest], m, k, n, rank, scale, dtype, workspace, workspace_bytes,
                    true};
  L.n_dest = n_dest;
  L.dest = y_dest;
  L.self_dest = self_dest;
  L.ldy = ldy;
  L.col0 = col0;
  if (w_scales != nullptr && !cfb::aligned_to(w_scales, 4)) return CF_ERR_MISALIGNED;
  return cfb::validate_and_run(L, stream);
}

size_t cf_rmsnorm_lora_linear_int8_workspace_bytes(int64_t m, int64_t k, int64_t rank) {
  return cfb::norm_linear_workspace(m, k, rank);
}

int cf_rmsnorm_lora_linear_int8(const void *x, const void *residual, const void *norm_weight,
                                float eps, const int8_t *w_codes, const float *w_scales,
                                const void *a, int a_layout, const void *b, int b_layout, void *y,
                                void *residual_out, int64_t m, int64_t k, int64_t n, int64_t rank,
                                float scale, int dtype, void *workspace, size_t workspace_bytes,
                                cf_stream_t stream) {
  using namespace cfb;
  if (m < 0 || k < 0 || n < 0) return CF_ERR_INVALID_ARGUMENT;
  if (m == 0 || n == 0) return CF_OK;
  if (x == nullptr || norm_weight == nullptr || (residual == nullptr) != (residual_out == nullptr)) {
    return CF_ERR_INVALID_ARGUMENT;
  }
  if (dtype != CF_DTYPE_BF16 && dtype != CF_DTYPE_F16) return CF_ERR_UNSUPPORTED;
  if (a_layout != CF_LAYOUT_REF && a_layout != CF_LAYOUT_T) return CF_ERR_INVALID_ARGUMENT;
  if (rank != 16 && rank != 32 && rank != 64) return CF_ERR_UNSUPPORTED;
  if (workspace == nullptr || workspace_bytes < norm_linear_workspace(m, k, rank)) {
    return CF_ERR_WORKSPACE;
  }
  if (!aligned_to(workspace, 256) || !aligned_to(norm_weight, 16)) return CF_ERR_MISALIGNED;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  const size_t p_bytes = cfb::workspace_bytes(m, rank, 2);
  if (m <= 128 || k % kBK != 0) {
    // Short token counts run on the decode kernel: normalise into the
    // workspace, then the plain W8 linear.
    void *normed = ws;
    if (int st = cf_fused_residual_rmsnorm(x, residual, norm_weight, dtype, normed, residual_out,
                                           m, k, eps, dtype, stream)) {
      return st;
    }
    return cf_lora_linear_int8(normed, w_codes, w_scales, a, a_layout, b, b_layout, y, m, k, n,
                               rank, scale, dtype, ws + align256(static_cast<size_t>(m * k) * 2),
                               p_bytes, stream);
  }
  float *row_scale = reinterpret_cast<float *>(ws);
  float *w32 = reinterpret_cast<float *>(ws + align256(static_cast<size_t>(m) * 4));
  void *a_w = reinterpret_cast<uint8_t *>(w32) + align256(static_cast<size_t>(k) * 4);
  void *p_ws = static_cast<uint8_t *>(a_w) + align256(static_cast<size_t>(k * rank) * 2);
  if (int st = residual_rms_stats(x, residual, residual_out, row_scale, m, k, eps, dtype, s)) {
    return st;
  }
  const int64_t total = k * rank;
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>((total + 255) / 256, 1024));
  const int a_t = a_layout == CF_LAYOUT_T ? 1 : 0;
  if (dtype == CF_DTYPE_BF16) {
    weight_adapter_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(
        static_cast<const __nv_bfloat16 *>(a), a_t, static_cast<const __nv_bfloat16 *>(norm_weight),
        static_cast<__nv_bfloat16 *>(a_w), w32, k, rank);
  } else {
    weight_adapter_kernel<__half><<<grid, 256, 0, s>>>(
        static_cast<const __half *>(a), a_t, static_cast<const __half *>(norm_weight),
        static_cast<__half *>(a_w), w32, k, rank);
  }
  if (int st = check_launch()) return st;
  const void *h = residual != nullptr ? residual_out : x;
  cfb::LinearArgs L{h, w_codes, CF_LAYOUT_T, w_scales, a_w, CF_LAYOUT_REF, b, b_layout, y, m, k, n,
                    rank, scale, dtype, p_ws, p_bytes, true};
  L.norm_w = w32;
  L.row_scale = row_scale;
  if (w_scales != nullptr && !aligned_to(w_scales, 4)) return CF_ERR_MISALIGNED;
  return cfb::validate_and_run(L, stream);
}

int cf_lora_linear_int8_allgather_mc(const void *x, const int8_t *w_codes, const float *w_scales,
                                     const void *a, int a_layout, const void *b, int b_layout,
                                     void *y_local, void *y_multicast, int64_t ldy, int64_t col0,
                                     int64_t m, int64_t k, int64_t n, int64_t rank, float scale,
                                     int dtype, void *workspace, size_t workspace_bytes,
                                     cf_stream_t stream) {
  if (y_local == nullptr || y_multicast == nullptr) return CF_ERR_INVALID_ARGUMENT;
  if (!cfb::aligned_to(y_local, 16) || !cfb::aligned_to(y_multicast, 16)) return CF_ERR_MISALIGNED;
  if (ldy <= 0 || col0 < 0 || col0 + n > ldy) return CF_ERR_INVALID_ARGUMENT;
  if (ldy % 8 != 0 || col0 % 8 != 0 || ldy > INT32_MAX || n % 128 != 0) return CF_ERR_UNSUPPORTED;
  void *const dest[1] = {y_local};
  cfb::LinearArgs L{x, w_codes, CF_LAYOUT_T, w_scales, a, a_layout, b, b_layout,
                    y_local, m, k, n, rank, scale, dtype, workspace, workspace_bytes, true};
  L.n_dest = 1;
  L.dest = dest;
  L.self_dest = 0;
  L.ldy = ldy;
  L.col0 = col0;
  L.mc = y_multicast;
  if (w_scales != nullptr && !cfb::aligned_to(w_scales, 4)) return CF_ERR_MISALIGNED;
  return cfb::validate_and_run(L, stream);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Column-sharded W8 linear with the all-gather on the copy engines.
//
// The wide kernel stores this rank's columns into the local destination only
// and, as each tile's stores land, bumps the counter of its row group (at
// most kCeGroups groups of whole 512-token row blocks). One copy stream per
// peer waits on each group's counter with a stream wait-value operation and
// then copies that group's [rows, n] block into the peer's destination with a
// 2-D memcpy, so NVLink traffic runs on the copy engines while the SMs keep
// computing the next row groups. The SMs' tile loop never waits for a peer.
// ---------------------------------------------------------------------------
namespace cfb {
namespace {

constexpr int kCeGroups = 16;
constexpr size_t kCeCounterBytes = 256;  // kCeGroups 32-bit counters, padded
static_assert(kCeGroups * sizeof(unsigned) <= kCeCounterBytes, "counter area");

using StreamWaitValue32Fn = CUresult (*)(CUstream, CUdeviceptr, cuuint32_t, unsigned int);

StreamWaitValue32Fn wait_value_fn() {
  static std::atomic<StreamWaitValue32Fn> cached{nullptr};
  StreamWaitValue32Fn fn = cached.load(std::memory_order_acquire);
  if (fn != nullptr) return fn;
  void *sym = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint("cuStreamWaitValue32", &sym, cudaEnableDefault, &q) !=
          cudaSuccess ||
      q != cudaDriverEntryPointSuccess || sym == nullptr) {
    return nullptr;
  }
  fn = reinterpret_cast<StreamWaitValue32Fn>(sym);
  cached.store(fn, std::memory_order_release);
  return fn;
}

// Copy streams and events of one device, created on first use and kept for
// the life of the process. Calls on one device serialise their enqueueing on
// `mu` (the streams and events are shared).
struct CopyLanes {
  std::mutex mu;
  bool ready = false;
  cudaStream_t streams[kMaxOuts] = {};
  cudaEvent_t start = nullptr;
  cudaEvent_t finished[kMaxOuts] = {};
};

CopyLanes g_copy_lanes[64];

int copy_lanes(CopyLanes **out) {
  int dev = 0;
  CFB_TRY_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return CF_ERR_UNSUPPORTED;
  CopyLanes &lanes = g_copy_lanes[dev];
  std::lock_guard<std::mutex> lock(lanes.mu);
  if (!lanes.ready) {
    int lo = 0, hi = 0;
    CFB_TRY_CUDA(cudaDeviceGetStreamPriorityRange(&lo, &hi));
    for (int d = 0; d < kMaxOuts; ++d) {
      CFB_TRY_CUDA(cudaStreamCreateWithPriority(&lanes.streams[d], cudaStreamNonBlocking, hi));
      CFB_TRY_CUDA(cudaEventCreateWithFlags(&lanes.finished[d], cudaEventDisableTiming));
    }
    CFB_TRY_CUDA(cudaEventCreateWithFlags(&lanes.start, cudaEventDisableTiming));
    lanes.ready = true;
  }
  *out = &lanes;
  return CF_OK;
}

}  // namespace
}  // namespace cfb

size_t cf_lora_linear_int8_allgather_ce_workspace_bytes(int64_t m, int64_t rank) {
  if (m <= 0 || rank <= 0) return 0;
  return cfb::workspace_bytes(m, rank) + cfb::kCeCounterBytes;
}

int cf_lora_linear_int8_allgather_ce(const void *x, const int8_t *w_codes, const float *w_scales,
                                     const void *a, int a_layout, const void *b, int b_layout,
                                     int n_dest, void *const *y_dest, int self_dest, int64_t ldy,
                                     int64_t col0, int64_t m, int64_t k, int64_t n, int64_t rank,
                                     float scale, int dtype, void *workspace,
                                     size_t workspace_bytes, cf_stream_t stream) {
  using namespace cfb;
  if (n_dest < 1 || n_dest > kMaxOuts || y_dest == nullptr) return CF_ERR_INVALID_ARGUMENT;
  if (self_dest < 0 || self_dest >= n_dest) return CF_ERR_INVALID_ARGUMENT;
  for (int d = 0; d < n_dest; ++d) {
    if (y_dest[d] == nullptr) return CF_ERR_INVALID_ARGUMENT;
    if (!aligned_to(y_dest[d], 16)) return CF_ERR_MISALIGNED;
  }
  if (m < 0 || n < 0) return CF_ERR_INVALID_ARGUMENT;
  if (ldy <= 0 || col0 < 0 || col0 + n > ldy) return CF_ERR_INVALID_ARGUMENT;
  if (ldy % 8 != 0 || col0 % 8 != 0 || ldy > INT32_MAX || n % 128 != 0) return CF_ERR_UNSUPPORTED;
  if (w_scales != nullptr && !aligned_to(w_scales, 4)) return CF_ERR_MISALIGNED;
  if (m == 0 || n == 0) return CF_OK;
  const size_t lin = cfb::workspace_bytes(m, rank);
  if (workspace == nullptr || workspace_bytes < lin + kCeCounterBytes) return CF_ERR_WORKSPACE;
  constexpr int kRowBlock = W8WideCfg<true>::BT;
  const int64_t n_rb = (m + kRowBlock - 1) / kRowBlock;
  const int rb_per_group = static_cast<int>((n_rb + kCeGroups - 1) / kCeGroups);
  const int n_groups = static_cast<int>((n_rb + rb_per_group - 1) / rb_per_group);
  const int64_t tiles_w = n / kBM;
  if (tiles_w * rb_per_group >= (1 << 24)) return CF_ERR_UNSUPPORTED;
  StreamWaitValue32Fn wait_value = wait_value_fn();
  if (wait_value == nullptr) return CF_ERR_UNSUPPORTED;
  CopyLanes *lanes = nullptr;
  if (int st = copy_lanes(&lanes)) return st;

  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  unsigned *done = reinterpret_cast<unsigned *>(static_cast<uint8_t *>(workspace) + lin);
  std::lock_guard<std::mutex> lock(lanes->mu);
  CFB_TRY_CUDA(cudaMemsetAsync(done, 0, kCeCounterBytes, s));
  CFB_TRY_CUDA(cudaEventRecord(lanes->start, s));
  LinearArgs L{x, w_codes, CF_LAYOUT_T, w_scales, a, a_layout, b, b_layout, y_dest[self_dest], m,
               k, n, rank, scale, dtype, workspace, lin, true};
  L.n_dest = 1;
  L.dest = y_dest + self_dest;
  L.ldy = ldy;
  L.col0 = col0;
  L.done = done;
  L.rb_per_group = rb_per_group;
  L.n_groups = n_groups;
  // Only enqueue waits once the kernel that releases them has launched.
  if (int st = validate_and_run(L, stream)) return st;

  const size_t pitch = static_cast<size_t>(ldy) * 2;
  const size_t width = static_cast<size_t>(n) * 2;
  for (int d = 0; d < n_dest; ++d) {
    if (d != self_dest) CFB_TRY_CUDA(cudaStreamWaitEvent(lanes->streams[d], lanes->start, 0));
  }
  for (int g = 0; g < n_groups; ++g) {
    const int64_t rb0 = static_cast<int64_t>(g) * rb_per_group;
    const int64_t rb1 = std::min<int64_t>(n_rb, rb0 + rb_per_group);
    const int64_t r0 = rb0 * kRowBlock;
    const int64_t r1 = std::min<int64_t>(m, rb1 * kRowBlock);
    const auto target = static_cast<cuuint32_t>(tiles_w * (rb1 - rb0));
    const size_t off = static_cast<size_t>(r0) * pitch + static_cast<size_t>(col0) * 2;
    const auto *src = static_cast<const uint8_t *>(y_dest[self_dest]) + off;
    for (int d = 0; d < n_dest; ++d) {
      if (d == self_dest) continue;
      const CUresult cr =
          wait_value(reinterpret_cast<CUstream>(lanes->streams[d]),
                     reinterpret_cast<CUdeviceptr>(done + g), target, CU_STREAM_WAIT_VALUE_GEQ);
      if (cr != CUDA_SUCCESS) return record_cuda_error(cudaErrorNotSupported);
      CFB_TRY_CUDA(cudaMemcpy2DAsync(static_cast<uint8_t *>(y_dest[d]) + off, pitch, src, pitch,
                                     width, static_cast<size_t>(r1 - r0),
                                     cudaMemcpyDeviceToDevice, lanes->streams[d]));
    }
  }
  for (int d = 0; d < n_dest; ++d) {
    if (d == self_dest) continue;
    CFB_TRY_CUDA(cudaEventRecord(lanes->finished[d], lanes->streams[d]));
    CFB_TRY_CUDA(cudaStreamWaitEvent(s, lanes->finished[d], 0));
  }
  return CF_OK;
}

int cf_matmul_f32(const float *a, const float *b, int b_layout, float *c, int64_t m, int64_t n,
                  int64_t k, int precise, cf_stream_t stream) {
  if (m < 0 || n < 0 || k < 0) return CF_ERR_INVALID_ARGUMENT;
  if (m == 0 || n == 0) return CF_OK;
  if (a == nullptr || b == nullptr || c == nullptr) return CF_ERR_INVALID_ARGUMENT;
  if (b_layout != CF_LAYOUT_REF && b_layout != CF_LAYOUT_T) return CF_ERR_INVALID_ARGUMENT;
  if (k == 0 || k % 4 != 0 || n % 4 != 0) return CF_ERR_UNSUPPORTED;
  if (m > INT32_MAX || n > INT32_MAX || k > INT32_MAX) return CF_ERR_UNSUPPORTED;
  for (const void *ptr : {static_cast<const void *>(a), static_cast<const void *>(b),
                          static_cast<const void *>(c)}) {
    if (!cfb::aligned_to(ptr, 16)) return CF_ERR_MISALIGNED;
  }
  return cfb::run_matmul_f32(a, b, b_layout, c, m, n, k, precise,
                             reinterpret_cast<cudaStream_t>(stream));
}

int cf_lora_merge_quantize_int8(const void *w, const void *lora_a, const void *lora_b,
                                int64_t n, int64_t k, int64_t rank, float scaling, int dtype,
                                int8_t *codes, float *scales, cf_stream_t stream) {
  if (n < 0 || k < 0 || rank < 0) return CF_ERR_INVALID_ARGUMENT;
  if (n == 0 || k == 0) return CF_OK;
  if (w == nullptr || lora_a == nullptr || lora_b == nullptr || codes == nullptr ||
      scales == nullptr) {
    return CF_ERR_INVALID_ARGUMENT;
  }
  if (dtype != CF_DTYPE_BF16 && dtype != CF_DTYPE_F16) return CF_ERR_UNSUPPORTED;
  if (rank != 16 && rank != 32 && rank != 64) return CF_ERR_UNSUPPORTED;
  if (k % cfb::kQuantBlockSize != 0 || n > INT32_MAX || k > INT32_MAX) return CF_ERR_UNSUPPORTED;
  for (const void *ptr : {w, lora_a, lora_b, static_cast<const void *>(codes)}) {
    if (!cfb::aligned_to(ptr, 16)) return CF_ERR_MISALIGNED;
  }
  if (!cfb::aligned_to(scales, 4)) return CF_ERR_MISALIGNED;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  return dtype == CF_DTYPE_BF16
             ? cfb::run_merge_quantize<true>(w, lora_a, lora_b, n, k, rank, scaling, codes,
                                             scales, s)
             : cfb::run_merge_quantize<false>(w, lora_a, lora_b, n, k, rank, scaling, codes,
                                              scales, s);
}

int cf_w8_swiglu_int8(const void *x, const int8_t *gate_codes, const float *gate_scales,
                      const int8_t *up_codes, const float *up_scales, void *y, int64_t m,
                      int64_t k, int64_t n, int dtype, cf_stream_t stream) {
  if (m < 0 || k < 0 || n < 0) return CF_ERR_INVALID_ARGUMENT;
  if (m == 0 || n == 0) return CF_OK;
  if (x == nullptr || gate_codes == nullptr || gate_scales == nullptr || up_codes == nullptr ||
      up_scales == nullptr || y == nullptr) {
    return CF_ERR_INVALID_ARGUMENT;
  }
  if (dtype != CF_DTYPE_BF16 && dtype != CF_DTYPE_F16) return CF_ERR_UNSUPPORTED;
  if (k == 0 || k % cfb::kQuantBlockSize != 0 || n % 8 != 0) return CF_ERR_UNSUPPORTED;
  if (m > INT32_MAX || n > INT32_MAX || k > INT32_MAX) return CF_ERR_UNSUPPORTED;
  for (const void *ptr : {x, static_cast<const void *>(gate_codes),
                          static_cast<const void *>(up_codes), static_cast<const void *>(y)}) {
    if (!cfb::aligned_to(ptr, 16)) return CF_ERR_MISALIGNED;
  }
  if (!cfb::aligned_to(gate_scales, 4) || !cfb::aligned_to(up_scales, 4)) return CF_ERR_MISALIGNED;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  return dtype == CF_DTYPE_BF16
             ? cfb::run_w8_swiglu<true>(x, gate_codes, gate_scales, up_codes, up_scales, y, m, k,
                                        n, s)
             : cfb::run_w8_swiglu<false>(x, gate_codes, gate_scales, up_codes, up_scales, y, m,
                                         k, n, s);
}
