// bf16 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM), fed by TMA.
//
//   D[m, n] = sum_k A[m, k] * B[n, k]        (A, B both K-major, fp32 accumulate)
//
// Used for every linear layer: with A = activations and B = weights it is the
// prefill GEMM (y = x W^T); with A = weights and B = activations ("swap-AB")
// the 128-row MMA M dimension runs over output features and the small token
// count becomes the MMA N dimension, which is how decode batches of 1..256
// tokens still use full 128xN tensor-core tiles. The epilogue writes D either
// as out[m][n] or transposed as out[n][m], optionally adding a residual.
//
// Structure (one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer: A/B tiles (128B-swizzled) into a STAGES-deep ring
//   warp 1      allocates TMEM; one elected lane issues tcgen05.mma (M=128,
//               N=BN, K=16) and tcgen05.commit to release smem stages and to
//               publish finished accumulators
//   warps 2-5   epilogue: tcgen05.ld (32 lanes x 16 columns) -> registers ->
//               bf16 global stores; double-buffered TMEM accumulators let the
//               epilogue of tile i overlap the MMAs of tile i+1
// Split-K (splits > 1) spreads the K loop of one output tile over several
// CTAs, so narrow decode GEMMs still put every SM on the weight stream. Each
// split writes its fp32 slice of the output ([split][rows][ldo], coalesced)
// and the kernel that consumes the output (fused add+RMSNorm, RoPE, ...) sums
// the slices while reading them: no in-kernel reduction tail, no atomics, a
// fixed summation order (deterministic).
//
// No TMA multicast anywhere (this kernel is also used on multi-GPU runs).
// All waits are bounded (fb_common.cuh).
#include "fb_common.cuh"

FB_DEFINE_STATUS

using namespace fbk;

namespace {

constexpr int BM = 128;
constexpr int BK = 64;  // 64 bf16 = 128 bytes = one swizzle row
constexpr int EPI_TRANSPOSE = 1;
constexpr int EPI_RESIDUAL = 2;
constexpr int EPI_A_STREAM = 4;  // L2 evict-first hint on A loads
constexpr int EPI_B_STREAM = 8;  // L2 evict-first hint on B loads
constexpr int NUM_THREADS = 192;

template <int BN>
struct Cfg {
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (200 * 1024) / STAGE_BYTES > 8 ? 8 : (200 * 1024) / STAGE_BYTES;
  static constexpr uint32_t TMEM_COLS = (2 * BN <= 32) ? 32 : (2 * BN <= 64) ? 64 : (2 * BN <= 128) ? 128 : (2 * BN <= 256) ? 256 : 512;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
};

template <int BN>
__device__ __forceinline__ void gemm_body(const CUtensorMap* tmA, const CUtensorMap* tmB, bf16* __restrict__ out,
                                          const bf16* residual, int M, int N, int K, int ldo, int mode, int splits,
                                          float* __restrict__ ws, long long split_stride) {
  using C = Cfg<BN>;
  constexpr int STAGES = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * C::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * C::STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_m = (M + BM - 1) / BM;
  const int num_n = (N + BN - 1) / BN;
  const int KB = (K + BK - 1) / BK;
  const int kb_per = (KB + splits - 1) / splits;
  const int num_tiles = num_m * num_n * splits;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 4);
    }
    *abort_flag = 0;
    fence_barrier_init();
    fence_proxy_async();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(tmA);
    tma_prefetch_desc(tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      const uint64_t pol_a = policy_evict_first();
      for (int t = blockIdx.x; t < num_tiles && !*(volatile int*)abort_flag; t += gridDim.x) {
        const int mn = t / splits, sp = t % splits;
        const int m_blk = mn % num_m, n_blk = mn / num_m;
        const int kb0 = sp * kb_per, kb1 = min(KB, kb0 + kb_per);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, FB_KERR_TIMEOUT_EMPTY)) {
            *(volatile int*)abort_flag = 1;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
          // Operands read exactly once per launch (decode weights) are hinted
          // evict-first so they do not push reused activations out of L2.
          if (mode & EPI_A_STREAM)
            tma_load_2d_hint(sA + stage * C::A_BYTES, tmA, &full[stage], kb * BK, m_blk * BM, pol_a);
          else
            tma_load_2d(sA + stage * C::A_BYTES, tmA, &full[stage], kb * BK, m_blk * BM);
          if (mode & EPI_B_STREAM)
            tma_load_2d_hint(sB + stage * C::B_BYTES, tmB, &full[stage], kb * BK, n_blk * BN, pol_a);
          else
            tma_load_2d(sB + stage * C::B_BYTES, tmB, &full[stage], kb * BK, n_blk * BN);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // Drain: every armed stage must complete before the CTA may exit.
      for (int s = 0; s < STAGES; ++s) {
        // The last phase armed on stage s completes when its consumer released it;
        // waiting on `empty` with the producer's parity covers both cases.
        mbar_wait(&empty[stage], phase ^ 1, FB_KERR_TIMEOUT_EMPTY);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16<BM, BN>();
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      for (int t = blockIdx.x; t < num_tiles && !*(volatile int*)abort_flag; t += gridDim.x, ++it) {
        const int sp = t % splits;
        const int kb0 = sp * kb_per, kb1 = min(KB, kb0 + kb_per);
        const int acc = it & 1;
        const uint32_t aphase = (it >> 1) & 1;
        if (!mbar_wait(&tempty[acc], aphase ^ 1, FB_KERR_TIMEOUT_TMEM)) {
          *(volatile int*)abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, FB_KERR_TIMEOUT_FULL)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t adesc = sdesc_sw128(smem_u32(sA + stage * C::A_BYTES));
          const uint64_t bdesc = sdesc_sw128(smem_u32(sB + stage * C::B_BYTES));
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            // +32 bytes per 16-element K step inside the 128-byte swizzle row.
            mma_bf16(d_tmem, adesc + (uint64_t)(k * 2), bdesc + (uint64_t)(k * 2), idesc,
                     (kb > kb0 || k > 0) ? 1u : 0u);
          }
          mma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        mma_commit(&tfull[acc]);
        if (!ok) {
          *(volatile int*)abort_flag = 1;
          break;
        }
      }
    }
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    const int row = quarter * 32 + lane;
    int it = 0;
    for (int t = blockIdx.x; t < num_tiles && !*(volatile int*)abort_flag; t += gridDim.x, ++it) {
      const int mn = t / splits, sp = t % splits;
      const int m_blk = mn % num_m, n_blk = mn / num_m;
      const int acc = it & 1;
      const uint32_t aphase = (it >> 1) & 1;
      if (!mbar_wait(&tfull[acc], aphase, FB_KERR_TIMEOUT_TMEM)) {
        *(volatile int*)abort_flag = 1;
        break;
      }
      tc_fence_after();
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * BN;
      const int gm = m_blk * BM + row;  // D row
      if (splits == 1) {
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 16) {
          uint32_t r[16];
          tmem_ld16(t_row + c0, r);
          tmem_ld_wait();
          const int gn0 = n_blk * BN + c0;
          if (gm < M) {
            if (mode & EPI_TRANSPOSE) {
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                const int gn = gn0 + i;
                if (gn < N) {
                  const size_t idx = static_cast<size_t>(gn) * ldo + gm;
                  float v = __uint_as_float(r[i]);
                  if (mode & EPI_RESIDUAL) v += bf2f(residual[idx]);
                  out[idx] = f2bf(v);
                }
              }
            } else {
              const size_t base = static_cast<size_t>(gm) * ldo + gn0;
              if (gn0 + 16 <= N) {
                float f[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) f[i] = __uint_as_float(r[i]);
                if (mode & EPI_RESIDUAL) {
                  float a[8], b[8];
                  unpack8(*reinterpret_cast<const uint4*>(residual + base), a);
                  unpack8(*reinterpret_cast<const uint4*>(residual + base + 8), b);
#pragma unroll
                  for (int i = 0; i < 8; ++i) {
                    f[i] += a[i];
                    f[8 + i] += b[i];
                  }
                }
                float lo[8], hi[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                  lo[i] = f[i];
                  hi[i] = f[8 + i];
                }
                *reinterpret_cast<uint4*>(out + base) = pack8(lo);
                *reinterpret_cast<uint4*>(out + base + 8) = pack8(hi);
              } else {
#pragma unroll
                for (int i = 0; i < 16; ++i)
                  if (gn0 + i < N) {
                    float v = __uint_as_float(r[i]);
                    if (mode & EPI_RESIDUAL) v += bf2f(residual[base + i]);
                    out[base + i] = f2bf(v);
                  }
              }
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[acc]);
      } else {
        // Split-K: write this split's fp32 slice of the output, in the output's
        // own layout ([split][rows][ldo]); the consuming kernel sums the slices.
        float* part = ws + static_cast<size_t>(sp) * split_stride;
        if (gm < M) {
#pragma unroll 1
          for (int c0 = 0; c0 < BN; c0 += 16) {
            uint32_t r[16];
            tmem_ld16(t_row + c0, r);
            tmem_ld_wait();
            const int gn0 = n_blk * BN + c0;
            if (mode & EPI_TRANSPOSE) {
#pragma unroll
              for (int i = 0; i < 16; ++i)
                if (gn0 + i < N) part[static_cast<size_t>(gn0 + i) * ldo + gm] = __uint_as_float(r[i]);
            } else if (gn0 + 16 <= N) {
              float4* dst = reinterpret_cast<float4*>(part + static_cast<size_t>(gm) * ldo + gn0);
#pragma unroll
              for (int i = 0; i < 4; ++i)
                dst[i] = make_float4(__uint_as_float(r[4 * i]), __uint_as_float(r[4 * i + 1]),
                                     __uint_as_float(r[4 * i + 2]), __uint_as_float(r[4 * i + 3]));
            } else {
#pragma unroll
              for (int i = 0; i < 16; ++i)
                if (gn0 + i < N) part[static_cast<size_t>(gm) * ldo + gn0 + i] = __uint_as_float(r[i]);
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[acc]);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, C::TMEM_COLS);
}

}  // namespace

#define FB_GEMM_INSTANCE(BN)                                                                                        \
  extern "C" __global__ void __launch_bounds__(NUM_THREADS, 1) fb_gemm_bf16_bn##BN(                                 \
      const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, bf16* out,                  \
      const bf16* residual, int M, int N, int K, int ldo, int mode, int splits, float* ws,                          \
      long long split_stride) {                                                                                      \
    gemm_body<BN>(&tmA, &tmB, out, residual, M, N, K, ldo, mode, splits, ws, split_stride);                        \
  }

FB_GEMM_INSTANCE(16)
FB_GEMM_INSTANCE(32)
FB_GEMM_INSTANCE(64)
FB_GEMM_INSTANCE(128)
FB_GEMM_INSTANCE(256)
