// Mixture-of-experts and block-scaled fp8 kernels (Qwen3-MoE family).
//
// Number format (the reference serves DeepSeek/Qwen "fp8 block" checkpoints):
//   weights      e4m3, one fp32 scale per 128 x 128 block     W = Wq * sw[o/128, k/128]
//   activations  e4m3, one fp32 scale per token per 128 dims  x = xq * sx[t, k/128]
//
// fb_moe_gemm_fp8_bn{32,64}: grouped GEMM over experts on tcgen05
//   (kind::f8f6f4, M = 128 weight rows, N = BN tokens, K = 32 per MMA).
//   A 128-wide K block is exactly one scale block, so every k-block's MMAs
//   write a fresh fp32 partial into TMEM (double-buffered) and the epilogue
//   warps promote it: acc[t] += partial[t] * sw * sx[t] (two-level
//   accumulation, fp32 throughout). Work units are (token chunk, 128-row
//   weight block) with the chunk table built on the device, so the launch
//   shape is static (CUDA-graph friendly) while expert loads vary per step.
//   Output is written transposed: out[row_start + t][o] (+ residual).
//   The same kernel with one "expert" is the dense fp8 linear layer.
//
// Routing: fb_moe_topk (softmax over experts, top-k, renormalise; warp per
//   token) -> fb_moe_plan (one CTA: per-expert counts, deterministic
//   expert-sorted positions, chunk table) -> fb_moe_dispatch_local (quantise
//   each token once, scatter its fp8 row to its k expert slots).
// After the experts: fb_moe_silu_mul_quant (gate/up -> fp8 activations for
//   the down projection) and fb_moe_combine_add_rmsnorm (top-k weighted sum
//   + residual + the next RMSNorm, one CTA per token).
//
// No TMA multicast; every wait bounded (fb_common.cuh).
#include <cuda_fp8.h>

#include "fb_common.cuh"

FB_DEFINE_STATUS

using namespace fbk;

namespace {

constexpr int NUM_THREADS = 192;
constexpr int QBLK = 128;       // scale block (tokens: 1 x 128, weights: 128 x 128)
constexpr float FP8_MAX = 448.f;
constexpr int EPI_RESIDUAL = 2;
constexpr int EPI_W_STREAM = 4;  // weights read once per launch: L2 evict-first
// Expert-parallel combine fused into the epilogue: row R of the output goes to
// rank (meta[R] >> 24), row (meta[R] & 0xFFFFFF) of that rank's combine buffer
// (`out` is the buffer's address in rank 0's window, `residual` the row map,
// peer_stride the byte distance between rank windows). Plain P2P stores.
constexpr int EPI_PEER_COMBINE = 32;
constexpr int MAX_KB = 32;       // K <= 4096
#ifndef FB_MOE_NBUF
#define FB_MOE_NBUF 8
#endif
// mode bits 12..15: L2 prefetch distance for weight tiles, in k-blocks (0 = off)
__device__ __forceinline__ int pf_dist(int mode) { return (mode >> 12) & 15; }

constexpr uint32_t tmem_cols_for(int cols) {
  return cols <= 32 ? 32 : cols <= 64 ? 64 : cols <= 128 ? 128 : cols <= 256 ? 256 : 512;
}

// kind::f8f6f4, A/B e4m3 (format 0), D f32, both K-major.
template <int M, int N>
__device__ __forceinline__ constexpr uint32_t idesc_e4m3() {
  return (1u << 4) | (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

__device__ __forceinline__ void mma_fp8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n}\n" ::
          "r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// 4 floats -> 4 e4m3 bytes (saturating, round to nearest even).
__device__ __forceinline__ uint32_t pack_e4m3x4(float a, float b, float c, float d) {
  const __nv_fp8x2_storage_t lo = __nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3);
  const __nv_fp8x2_storage_t hi = __nv_cvt_float2_to_fp8x2(make_float2(c, d), __NV_SATFINITE, __NV_E4M3);
  return static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
}

// Scale rows are padded to a multiple of 4 floats (16 bytes) so that the
// producer can fetch a unit's scales with one bulk copy.
__host__ __device__ constexpr int kb_pad(int kb) { return (kb + 3) & ~3; }

// Bulk (non-tensor) global -> shared copy, completion on `bar`. Both
// addresses 16-byte aligned, bytes a multiple of 16. No multicast.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// Resident CTAs per SM of the promote GEMM, per token-tile width. The
// per-k-block promotion chain (MMA commit -> TMEM load -> FMA -> release)
// bounds one CTA's rate, not HBM: at 32-token tiles three CTAs per SM
// stream the expert weights 1.5x faster than one (same bytes, same result);
// 64-token tiles gain nothing and keep the deeper single-CTA ring.
template <int BN>
struct MoeOcc {
  static constexpr int CTAS = BN == 32 ? 3 : 1;
};

template <int BN>
struct GemmCfg {
  static constexpr int CTAS = MoeOcc<BN>::CTAS;
  static constexpr int A_BYTES = 128 * QBLK;  // 128 weight rows x 128 K bytes
  static constexpr int B_BYTES = BN * QBLK;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int BUDGET = CTAS == 1 ? 200 * 1024 : CTAS == 2 ? 100 * 1024 : 60 * 1024;  // operand ring
  static constexpr int STAGES = BUDGET / STAGE_BYTES > 10 ? 10 : BUDGET / STAGE_BYTES;
  // TMEM partial buffers: the epilogue may lag the MMAs by NBUF - 1 k-blocks;
  // the resident CTAs share the SM's 512 columns (power-of-two allocations)
  static constexpr int CTA_COLS = CTAS == 1 ? 512 : CTAS == 2 ? 256 : 128;
  static constexpr int NBUF = FB_MOE_NBUF * BN > CTA_COLS ? CTA_COLS / BN : FB_MOE_NBUF;
  static constexpr uint32_t TMEM_COLS = tmem_cols_for(NBUF * BN);
  static constexpr int XS_FLOATS = BN * MAX_KB;  // token scales of one unit [BN][KBp]
};

// Work unit u = (chunk c, weight row block ob) with c = u % num_chunks.
// Warp 0 lane 0: per unit, one bulk copy of the unit's token scales
//   [BN][KBp] and weight scales [KBp] into scale slot (unit & 1), then the
//   TMA loads of the K loop; warp 1 lane 0: per k-block 4 MMAs into a fresh
//   TMEM partial (NBUF buffers); warps 2-5: per k-block promote the partial
//   with sw[kb] * sx[t][kb], per unit store the 128 x BN tile transposed.
// ssc[kb][t] = sw[kb] * sx[t][kb] for the unit's KB k-blocks (128 threads).
template <int BN>
__device__ __noinline__ void combine_scales(float* ssc, const float* xsu, const float* wsu, int KB, int KBp, int et) {
  for (int i = et; i < KB * BN; i += 128) {
    const int kb = i / BN, t = i - kb * BN;
    ssc[i] = xsu[t * KBp + kb] * wsu[kb];
  }
}

template <int BN>
__device__ __forceinline__ void moe_gemm_body(const CUtensorMap* tmW, const CUtensorMap* tmX,
                                              const float* __restrict__ w_scale, const float* __restrict__ x_scale,
                                              const int4* __restrict__ chunks, const int* __restrict__ meta,
                                              bf16* out, const bf16* residual, int O, int K, int ldo, int mode,
                                              long long peer_stride) {
  using C = GemmCfg<BN>;
  constexpr int STAGES = C::STAGES;
  constexpr int NBUF = C::NBUF;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * C::A_BYTES;
  float* sxs = reinterpret_cast<float*>(smem + STAGES * C::STAGE_BYTES);  // [2][BN * KBp]
  float* sws = sxs + 2 * C::XS_FLOATS;                                       // [2][MAX_KB]
  float* ssc = sws + 2 * MAX_KB;  // [MAX_KB][BN]: sw[kb] * sx[t][kb] of the unit being promoted
  uint64_t* full = reinterpret_cast<uint64_t*>(ssc + MAX_KB * BN);
  uint64_t* empty = full + STAGES;
  uint64_t* pfull = empty + STAGES;
  uint64_t* pempty = pfull + NBUF;
  uint64_t* sfull = pempty + NBUF;
  uint64_t* sempty = sfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sempty + 2);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int KB = K / QBLK;
  const int KBp = kb_pad(KB);
  const int num_ob = O / 128;
  const int num_chunks = meta[0];
  const int num_units = num_chunks * num_ob;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < NBUF; ++a) {
      mbar_init(&pfull[a], 1);
      mbar_init(&pempty[a], 4);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&sfull[a], 1);
      mbar_init(&sempty[a], 4);
    }
    *abort_flag = (KB > MAX_KB || (K % QBLK) || (O % 128)) ? 1 : 0;
    if (*abort_flag) set_status(FB_KERR_BAD_ARG);
    fence_barrier_init();
    fence_proxy_async();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(tmW);
    tma_prefetch_desc(tmX);
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
    // ---------------- producer: scales (bulk copy) + operand tiles (TMA) ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      const uint64_t pol = policy_evict_first();
      uint32_t j = 0;  // units of this CTA
      for (int u = blockIdx.x; u < num_units && !*(volatile int*)abort_flag; u += gridDim.x, ++j) {
        const int c = u % num_chunks, ob = u / num_chunks;
        const int4 ch = chunks[c];
        const int wrow = ch.x * O + ob * 128;
        const uint32_t slot = j & 1;
        if (!mbar_wait(&sempty[slot], ((j >> 1) & 1) ^ 1, FB_KERR_TIMEOUT_EMPTY)) {
          *(volatile int*)abort_flag = 1;
          break;
        }
        const uint32_t xs_bytes = BN * KBp * 4, ws_bytes = KBp * 4;
        const int pf = pf_dist(mode);
        for (int kb = 0; kb < min(pf, KB); ++kb) tma_prefetch_2d(tmW, kb * QBLK, wrow);
        mbar_arrive_expect_tx(&sfull[slot], xs_bytes + ws_bytes);
        bulk_load(sxs + slot * C::XS_FLOATS, x_scale + static_cast<size_t>(ch.y) * KBp, xs_bytes, &sfull[slot]);
        bulk_load(sws + slot * MAX_KB, w_scale + (static_cast<size_t>(ch.x) * num_ob + ob) * KBp, ws_bytes,
                  &sfull[slot]);
        for (int kb = 0; kb < KB; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, FB_KERR_TIMEOUT_EMPTY)) {
            *(volatile int*)abort_flag = 1;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
          const int kx = kb * QBLK;
          if (pf && kb + pf < KB) tma_prefetch_2d(tmW, (kb + pf) * QBLK, wrow);
          if (mode & EPI_W_STREAM)
            tma_load_2d_hint(sA + stage * C::A_BYTES, tmW, &full[stage], kx, wrow, pol);
          else
            tma_load_2d(sA + stage * C::A_BYTES, tmW, &full[stage], kx, wrow);
          tma_load_2d(sB + stage * C::B_BYTES, tmX, &full[stage], kx, ch.y);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // Drain: every armed operand stage and scale slot completes before exit.
      for (int s = 0; s < STAGES; ++s) {
        mbar_wait(&empty[stage], phase ^ 1, FB_KERR_TIMEOUT_EMPTY);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
      for (int s = 0; s < 2; ++s, ++j) mbar_wait(&sempty[j & 1], ((j >> 1) & 1) ^ 1, FB_KERR_TIMEOUT_EMPTY);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer: one fresh partial per k-block ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_e4m3<128, BN>();
      int stage = 0;
      uint32_t phase = 0;
      uint32_t g = 0;  // partials issued by this CTA
      for (int u = blockIdx.x; u < num_units && !*(volatile int*)abort_flag; u += gridDim.x) {
        bool ok = true;
        for (int kb = 0; kb < KB; ++kb, ++g) {
          const uint32_t buf = g % NBUF;
          if (!mbar_wait(&pempty[buf], ((g / NBUF) & 1) ^ 1, FB_KERR_TIMEOUT_TMEM) ||
              !mbar_wait(&full[stage], phase, FB_KERR_TIMEOUT_FULL)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t adesc = sdesc_sw128(smem_u32(sA + stage * C::A_BYTES));
          const uint64_t bdesc = sdesc_sw128(smem_u32(sB + stage * C::B_BYTES));
#pragma unroll
          for (int k = 0; k < QBLK / 32; ++k)  // +32 bytes per 32-element K step
            mma_fp8(tmem_base + buf * BN, adesc + (uint64_t)(k * 2), bdesc + (uint64_t)(k * 2), idesc,
                    k > 0 ? 1u : 0u);
          mma_commit(&empty[stage]);
          mma_commit(&pfull[buf]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) {
          *(volatile int*)abort_flag = 1;
          break;
        }
      }
    }
  } else {
    // ---------------- epilogue (warps 2..5): promote + store ----------------
    const int quarter = warp & 3;
    uint32_t g = 0, j = 0;
    for (int u = blockIdx.x; u < num_units && !*(volatile int*)abort_flag; u += gridDim.x, ++j) {
      const int c = u % num_chunks, ob = u / num_chunks;
      const int4 ch = chunks[c];
      const uint32_t slot = j & 1;
      if (!mbar_wait(&sfull[slot], (j >> 1) & 1, FB_KERR_TIMEOUT_FULL)) {
        *(volatile int*)abort_flag = 1;
        break;
      }
      const float* xsu = sxs + slot * C::XS_FLOATS;
      const float* wsu = sws + slot * MAX_KB;
      // One combined scale per (k-block, token), laid out k-block-major (one
      // broadcast load and one FMA per token in the promote): the four epilogue warps
      // first wait for each other (the previous unit's promote is done with
      // ssc), fill it, and wait again. The scale slot is free after that.
      asm volatile("bar.sync 1, 128;" ::: "memory");
      combine_scales<BN>(ssc, xsu, wsu, KB, KBp, threadIdx.x - 64);
      asm volatile("bar.sync 1, 128;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&sempty[slot]);
      float acc[BN];
#pragma unroll
      for (int t = 0; t < BN; ++t) acc[t] = 0.f;
      bool ok = true;
      for (int kb = 0; kb < KB; ++kb, ++g) {
        const uint32_t buf = g % NBUF;
        if (!mbar_wait(&pfull[buf], (g / NBUF) & 1, FB_KERR_TIMEOUT_TMEM)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t r[BN];
        const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + buf * BN;
#pragma unroll
        for (int c0 = 0; c0 < BN; c0 += 16) tmem_ld16(taddr + c0, *reinterpret_cast<uint32_t(*)[16]>(&r[c0]));
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&pempty[buf]);
        const float* sc = ssc + kb * BN;
#pragma unroll
        for (int t = 0; t < BN; ++t) acc[t] = fmaf(__uint_as_float(r[t]), sc[t], acc[t]);
      }
      if (!ok) {
        *(volatile int*)abort_flag = 1;
        break;
      }
      const int o = ob * 128 + quarter * 32 + lane;
      if (mode & EPI_PEER_COMBINE) {
        const int* rowmap = reinterpret_cast<const int*>(residual);
#pragma unroll
        for (int t = 0; t < BN; ++t) {
          if (t < ch.z) {
            const int m = rowmap[ch.y + t];
            bf16* dst = reinterpret_cast<bf16*>(reinterpret_cast<char*>(out) + static_cast<long long>(m >> 24) * peer_stride);
            dst[static_cast<size_t>(m & 0xFFFFFF) * ldo + o] = f2bf(acc[t]);
          }
        }
        continue;
      }
#pragma unroll
      for (int t = 0; t < BN; ++t) {
        if (t < ch.z) {
          const size_t idx = static_cast<size_t>(ch.y + t) * ldo + o;
          float v = acc[t];
          if (mode & EPI_RESIDUAL) v += bf2f(residual[idx]);
          out[idx] = f2bf(v);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, C::TMEM_COLS);
}

}  // namespace

#define FB_MOE_GEMM_INSTANCE(BN)                                                                                    \
  extern "C" __global__ void __launch_bounds__(NUM_THREADS, MoeOcc<BN>::CTAS) fb_moe_gemm_fp8_bn##BN(                             \
      const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX, const float* w_scale,       \
      const float* x_scale, const int4* chunks, const int* meta, bf16* out, const bf16* residual, int O, int K,     \
      int ldo, int mode, long long peer_stride) {                                                                    \
    pdl_entry();                                                                                                    \
    moe_gemm_body<BN>(&tmW, &tmX, w_scale, x_scale, chunks, meta, out, residual, O, K, ldo, mode, peer_stride);     \
  }

FB_MOE_GEMM_INSTANCE(32)
FB_MOE_GEMM_INSTANCE(64)

// ---- routing -----------------------------------------------------------------------------
// logits [T, E] bf16 (row stride ld); E % 32 == 0, E <= 256; topk <= 8.
// Softmax over E, top-k (ties -> lower expert index), optional renormalisation
// of the k probabilities. One warp per token.
extern "C" __global__ void __launch_bounds__(256) fb_moe_topk(const bf16* __restrict__ logits, int ld, int T, int E,
                                                             int topk, int renorm, int* __restrict__ ids,
                                                             float* __restrict__ weights) {
  pdl_entry();
  const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  const int per = E / 32;
  float v[8];
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    v[i] = i < per ? bf2f(logits[static_cast<size_t>(t) * ld + i * 32 + lane]) : -INFINITY;
    mx = fmaxf(mx, v[i]);
  }
  mx = warp_max(mx);
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    v[i] = i < per ? expf(v[i] - mx) : -1.f;  // -1: never selected
    s += i < per ? v[i] : 0.f;
  }
  s = warp_sum(s);
  const float inv = 1.f / s;
  float sel_sum = 0.f;
  float my_w = 0.f;
  int my_id = 0;
  for (int k = 0; k < topk; ++k) {
    float best = -1.f;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int e = i * 32 + lane;
      if (v[i] > best || (v[i] == best && e < bi)) {
        best = v[i];
        bi = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ob > best || (ob == best && oi < bi)) {
        best = ob;
        bi = oi;
      }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if ((bi & 31) == lane && (bi >> 5) == i) v[i] = -2.f;  // taken
    const float p = best * inv;
    sel_sum += p;
    if (lane == k) {
      my_w = p;
      my_id = bi;
    }
  }
  if (lane < topk) {
    ids[t * topk + lane] = my_id;
    weights[t * topk + lane] = renorm ? my_w / sel_sum : my_w;
  }
}

// One CTA of 1024 threads. ids [P] (P = T * topk pairs) -> per-expert counts,
// expert-sorted position of every pair (stable: pair order within an expert),
// the chunk table {expert, first row, rows, 0} with chunks of <= bn rows, and
// meta = {num_chunks, P}. Warp w owns the pairs [w * S, (w + 1) * S):
// (1) each warp counts its pairs per expert (match_any leaders, in order);
// (2) per expert, a shuffle scan over the 32 warps gives each warp its first
//     row inside the expert, and the total is the expert's count;
// (3) warp 0 scans counts and chunk counts over the experts;
// (4) each warp walks its pairs again and assigns positions in order.
extern "C" __global__ void __launch_bounds__(1024) fb_moe_plan(const int* __restrict__ ids, int P, int E, int bn,
                                                              int* __restrict__ pos, int* __restrict__ counts,
                                                              int4* __restrict__ chunks, int* __restrict__ meta) {
  pdl_entry();
  __shared__ int cnt[256], off[256], coff[256];
  __shared__ int wbase[32][257];  // [warp][expert]; odd stride: the scan in (2) reads a column
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (E > 256) {
    if (tid == 0) set_status(FB_KERR_BAD_ARG);
    return;
  }
  for (int i = tid; i < 32 * E; i += 1024) wbase[i / E][i % E] = 0;
  __syncthreads();
  const int S = ((P + 31) / 32 + 31) / 32 * 32;  // pairs per warp, whole 32-pair rounds
  const int p0 = warp * S, p1 = min(P, p0 + S);
  const unsigned lt = (1u << lane) - 1;
  for (int b = p0; b < p1; b += 128) {
    int ev[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int p = b + u * 32 + lane;
      ev[u] = p < p1 ? ids[p] : -1;
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const unsigned same = __match_any_sync(0xffffffffu, ev[u]);
      if (ev[u] >= 0 && (same & lt) == 0) wbase[warp][ev[u]] += __popc(same);
      __syncwarp();
    }
  }
  __syncthreads();
  for (int e = warp; e < E; e += 32) {
    const int v = wbase[lane][e];
    int inc = v;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, inc, d);
      if (lane >= d) inc += n;
    }
    wbase[lane][e] = inc - v;
    if (lane == 31) cnt[e] = inc;
  }
  __syncthreads();
  if (warp == 0) {
    int c[8], sa = 0, sb = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int e = lane * 8 + i;
      c[i] = e < E ? cnt[e] : 0;
      sa += c[i];
      sb += (c[i] + bn - 1) / bn;
    }
    int ia = sa, ib = sb;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int na = __shfl_up_sync(0xffffffffu, ia, d);
      const int nb = __shfl_up_sync(0xffffffffu, ib, d);
      if (lane >= d) {
        ia += na;
        ib += nb;
      }
    }
    int ea = ia - sa, eb = ib - sb;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int e = lane * 8 + i;
      if (e < E) {
        off[e] = ea;
        coff[e] = eb;
      }
      ea += c[i];
      eb += (c[i] + bn - 1) / bn;
    }
    if (lane == 31) {
      meta[0] = ib;
      meta[1] = P;
    }
  }
  __syncthreads();
  for (int e = tid; e < E; e += 1024) {
    counts[e] = cnt[e];
    const int n = cnt[e];
    for (int j = 0, r = 0; r < n; ++j, r += bn) chunks[coff[e] + j] = make_int4(e, off[e] + r, min(bn, n - r), 0);
  }
  for (int b = p0; b < p1; b += 128) {
    int ev[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int p = b + u * 32 + lane;
      ev[u] = p < p1 ? ids[p] : -1;
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const unsigned same = __match_any_sync(0xffffffffu, ev[u]);
      const int rank = __popc(same & lt);
      if (ev[u] >= 0) pos[b + u * 32 + lane] = off[ev[u]] + wbase[warp][ev[u]] + rank;
      __syncwarp();
      if (ev[u] >= 0 && rank == 0) wbase[warp][ev[u]] += __popc(same);
      __syncwarp();
    }
  }
}

// Quantise token rows to e4m3 with one scale per 128 dims and scatter each
// row to its k destinations: xq[pos[t * k + j]] (pos == nullptr: row t).
// One warp per (token, group of 4 scale blocks); H % 128 == 0.
extern "C" __global__ void __launch_bounds__(256) fb_moe_dispatch_local(const bf16* __restrict__ x, int ldx, int T,
                                                                       int H, const int* __restrict__ pos, int topk,
                                                                       uint8_t* __restrict__ xq,
                                                                       float* __restrict__ xs) {
  pdl_entry();
  constexpr int BPW = 4;
  const int nb = H / QBLK;
  const int groups = (nb + BPW - 1) / BPW;
  const int w = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (w >= T * groups) return;
  const int t = w / groups, b0 = (w % groups) * BPW;
  uint32_t q[BPW];
  float sc[BPW];
#pragma unroll
  for (int i = 0; i < BPW; ++i) {
    const int b = b0 + i;
    if (b >= nb) break;
    const uint2 raw = *reinterpret_cast<const uint2*>(x + static_cast<size_t>(t) * ldx + b * QBLK + lane * 4);
    const float2 f0 = __bfloat1622float2(*reinterpret_cast<const bf162*>(&raw.x));
    const float2 f1 = __bfloat1622float2(*reinterpret_cast<const bf162*>(&raw.y));
    const float am = warp_max(fmaxf(fmaxf(fabsf(f0.x), fabsf(f0.y)), fmaxf(fabsf(f1.x), fabsf(f1.y))));
    const float s = fmaxf(am, 1e-12f) / FP8_MAX;
    const float inv = 1.f / s;
    q[i] = pack_e4m3x4(f0.x * inv, f0.y * inv, f1.x * inv, f1.y * inv);
    sc[i] = s;
  }
  for (int j = 0; j < (pos ? topk : 1); ++j) {
    const int row = pos ? pos[t * topk + j] : t;
    uint32_t* dst = reinterpret_cast<uint32_t*>(xq + static_cast<size_t>(row) * H);
#pragma unroll
    for (int i = 0; i < BPW; ++i) {
      const int b = b0 + i;
      if (b >= nb) break;
      dst[b * 32 + lane] = q[i];
      if (lane == i) xs[static_cast<size_t>(row) * kb_pad(nb) + b] = sc[i];
    }
  }
}

// gu [rows, 2I] bf16 (gate | up) -> act = silu(gate) * up as e4m3 [rows, I]
// with one scale per 128 features. One warp per row; I % 128 == 0.
extern "C" __global__ void __launch_bounds__(256) fb_moe_silu_mul_quant(const bf16* __restrict__ gu, int rows, int I,
                                                                       const int* __restrict__ meta,
                                                                       uint8_t* __restrict__ aq,
                                                                       float* __restrict__ as) {
  pdl_entry();
  const int r = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int n = meta ? min(rows, meta[1]) : rows;
  if (r >= n) return;
  const int nb = I / QBLK;
  const bf16* g = gu + static_cast<size_t>(r) * 2 * I;
  for (int b = 0; b < nb; ++b) {
    const uint2 rg = *reinterpret_cast<const uint2*>(g + b * QBLK + lane * 4);
    const uint2 ru = *reinterpret_cast<const uint2*>(g + I + b * QBLK + lane * 4);
    const float2 g0 = __bfloat1622float2(*reinterpret_cast<const bf162*>(&rg.x));
    const float2 g1 = __bfloat1622float2(*reinterpret_cast<const bf162*>(&rg.y));
    const float2 u0 = __bfloat1622float2(*reinterpret_cast<const bf162*>(&ru.x));
    const float2 u1 = __bfloat1622float2(*reinterpret_cast<const bf162*>(&ru.y));
    float a[4] = {g0.x, g0.y, g1.x, g1.y};
    const float u[4] = {u0.x, u0.y, u1.x, u1.y};
    float am = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      a[i] = a[i] / (1.f + __expf(-a[i])) * u[i];
      am = fmaxf(am, fabsf(a[i]));
    }
    am = warp_max(am);
    const float s = fmaxf(am, 1e-12f) / FP8_MAX;
    const float inv = 1.f / s;
    reinterpret_cast<uint32_t*>(aq + static_cast<size_t>(r) * I)[b * 32 + lane] =
        pack_e4m3x4(a[0] * inv, a[1] * inv, a[2] * inv, a[3] * inv);
    if (lane == 0) as[static_cast<size_t>(r) * kb_pad(nb) + b] = s;
  }
}

// h[t] += sum_j w[t, j] * y[pos[t * k + j]]; x[t] = rmsnorm(h[t]) * norm_w.
// One CTA of 256 threads per token, 8 features per thread; H = 2048 exactly
// 256 x 8 (any H % 8 == 0, H <= 4096 works with the loop).
extern "C" __global__ void __launch_bounds__(256) fb_moe_combine_add_rmsnorm(
    const bf16* __restrict__ y, int ldy, const int* __restrict__ pos, const float* __restrict__ w, int topk,
    bf16* __restrict__ h, const bf16* __restrict__ norm_w, bf16* __restrict__ x, int T, int H, float eps) {
  pdl_entry();
  const int t = blockIdx.x;
  __shared__ float red[8];
  float acc[2][8] = {};
  float ss = 0.f;
#pragma unroll
  for (int nv = 0; nv < 2; ++nv) {
    const int c = threadIdx.x * 8 + nv * 2048;
    if (c >= H) break;
    float a[8];
    unpack8(*reinterpret_cast<const uint4*>(h + static_cast<size_t>(t) * H + c), a);
    for (int j = 0; j < topk; ++j) {
      const int row = pos[t * topk + j];
      const float wj = w[t * topk + j];
      float b[8];
      unpack8(*reinterpret_cast<const uint4*>(y + static_cast<size_t>(row) * ldy + c), b);
#pragma unroll
      for (int i = 0; i < 8; ++i) a[i] = fmaf(wj, b[i], a[i]);
    }
    // round through bf16 like every other residual update
    const uint4 hv = pack8(a);
    *reinterpret_cast<uint4*>(h + static_cast<size_t>(t) * H + c) = hv;
    unpack8(hv, acc[nv]);
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += acc[nv][i] * acc[nv][i];
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) tot += red[i];
  const float rs = rsqrtf(tot / H + eps);
#pragma unroll
  for (int nv = 0; nv < 2; ++nv) {
    const int c = threadIdx.x * 8 + nv * 2048;
    if (c >= H) break;
    float g[8], o[8];
    unpack8(*reinterpret_cast<const uint4*>(norm_w + c), g);
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = acc[nv][i] * rs * g[i];
    *reinterpret_cast<uint4*>(x + static_cast<size_t>(t) * H + c) = pack8(o);
  }
}

// Block quantisation of a bf16 matrix [R, C] (R, C multiples of 128) to e4m3
// with one fp32 scale per 128 x 128 block: scales [R/128, C/128]. One CTA per block.
extern "C" __global__ void __launch_bounds__(256) fb_quant_block_fp8(const bf16* __restrict__ w, int R, int Cc,
                                                                    uint8_t* __restrict__ q,
                                                                    float* __restrict__ scales) {
  pdl_entry();
  const int bc = blockIdx.x, br = blockIdx.y;
  __shared__ float red[8];
  float am = 0.f;
  // 128 rows x 128 cols: thread -> rows (tid / 16) + 16 i, cols (tid % 16) * 8 .. +8
  const int r0 = threadIdx.x / 16, c0 = (threadIdx.x % 16) * 8;
  float v[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const size_t row = static_cast<size_t>(br) * 128 + r0 + 16 * i;
    unpack8(*reinterpret_cast<const uint4*>(w + row * Cc + bc * 128 + c0), v[i]);
#pragma unroll
    for (int j = 0; j < 8; ++j) am = fmaxf(am, fabsf(v[i][j]));
  }
  am = warp_max(am);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = am;
  __syncthreads();
  float m = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) m = fmaxf(m, red[i]);
  const float s = fmaxf(m, 1e-12f) / FP8_MAX;
  const float inv = 1.f / s;
  if (threadIdx.x == 0) scales[static_cast<size_t>(br) * kb_pad(Cc / 128) + bc] = s;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const size_t row = static_cast<size_t>(br) * 128 + r0 + 16 * i;
    uint2 o;
    o.x = pack_e4m3x4(v[i][0] * inv, v[i][1] * inv, v[i][2] * inv, v[i][3] * inv);
    o.y = pack_e4m3x4(v[i][4] * inv, v[i][5] * inv, v[i][6] * inv, v[i][7] * inv);
    *reinterpret_cast<uint2*>(q + row * Cc + bc * 128 + c0) = o;
  }
}

// Random block-scaled e4m3 weights without a bf16 staging copy: element
// (r, c) of the [R, C] matrix is N(0, std) from the counter-based stream
// (seed, pair ((r + row_offset) * C + c) / 2), then the 128 x 128 block is
// quantised as in fb_quant_block_fp8. row_offset lets a shard (e.g. this
// rank's experts) draw the same values as the full matrix. One CTA per block.
extern "C" __global__ void __launch_bounds__(256) fb_init_fp8_block(uint8_t* __restrict__ q, float* __restrict__ scales,
                                                                   int R, int Cc, unsigned long long seed, float std,
                                                                   long long row_offset) {
  pdl_entry();
  const int bc = blockIdx.x, br = blockIdx.y;
  __shared__ float red[8];
  const int r0 = threadIdx.x / 16, c0 = (threadIdx.x % 16) * 8;
  float v[8][8];
  float am = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint64_t row = static_cast<uint64_t>(br) * 128 + r0 + 16 * i + row_offset;
    const uint64_t e0 = row * static_cast<uint64_t>(Cc) + bc * 128 + c0;  // even
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 z = rng_normal2(seed, e0 / 2 + j);
      v[i][2 * j] = std * z.x;
      v[i][2 * j + 1] = std * z.y;
      am = fmaxf(am, fmaxf(fabsf(v[i][2 * j]), fabsf(v[i][2 * j + 1])));
    }
  }
  am = warp_max(am);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = am;
  __syncthreads();
  float m = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) m = fmaxf(m, red[i]);
  const float s = fmaxf(m, 1e-12f) / FP8_MAX;
  const float inv = 1.f / s;
  if (threadIdx.x == 0) scales[static_cast<size_t>(br) * kb_pad(Cc / 128) + bc] = s;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const size_t row = static_cast<size_t>(br) * 128 + r0 + 16 * i;
    uint2 o;
    o.x = pack_e4m3x4(v[i][0] * inv, v[i][1] * inv, v[i][2] * inv, v[i][3] * inv);
    o.y = pack_e4m3x4(v[i][4] * inv, v[i][5] * inv, v[i][6] * inv, v[i][7] * inv);
    *reinterpret_cast<uint2*>(q + row * Cc + bc * 128 + c0) = o;
  }
}

// Dense layers as a one-"expert" grouped GEMM: chunk table of ceil(T / bn)
// chunks over rows [0, T) with meta = {chunks, T}. One thread per chunk.
extern "C" __global__ void fb_moe_dense_chunks(int T, int bn, int4* __restrict__ chunks, int* __restrict__ meta) {
  pdl_entry();
  const int n = (T + bn - 1) / bn;
  for (int c = threadIdx.x; c < n; c += blockDim.x) chunks[c] = make_int4(0, c * bn, min(bn, T - c * bn), 0);
  if (threadIdx.x == 0) {
    meta[0] = n;
    meta[1] = T;
  }
}

// ==== weight-only fp8: e4m3 block-scaled weights x bf16 activations ===================
//
// fb_moe_gemm_w8_bn{32,64,128}: the grouped / dense GEMM of the fp8 checkpoints
// with the weights dequantised on chip. Per k-block (128 K):
//   warp 0      TMA: e4m3 weight tile [128 x 128 B] + bf16 activation tile
//               [BN x 128] (two 64-wide boxes) into a ring stage; per unit a
//               bulk copy of the unit's weight scales
//   warps 2-5   converters: thread r turns weight row r into bf16,
//               w = e4m3 * sw[kb] (exact e4m3 -> bf16 bit move, one bf16x2
//               multiply per pair), written in the 128B-swizzled K-major
//               layout the MMA reads; fence.proxy.async; release
//   warp 1      MMA: 8 x tcgen05.mma kind::f16 (M = 128, N = BN, K = 16)
//               accumulating the whole K loop in TMEM (no promotion)
//   warps 6-9   epilogue once per unit: TMEM -> bf16, transposed store (+ residual)
// HBM traffic is the fp8 weights (half of bf16); the tensor core runs bf16.
namespace {

constexpr int W8_THREADS = 320;
constexpr int W8_CBUF = 2;  // converted (bf16) weight tiles in flight

template <int BN>
struct W8Cfg {
  static constexpr int A8_BYTES = 128 * 128;         // e4m3 weight tile
  static constexpr int B_BYTES = BN * 128 * 2;        // bf16 activations, two 64-wide halves
  static constexpr int STAGE_BYTES = A8_BYTES + B_BYTES;
  static constexpr int C_BYTES = 128 * 128 * 2;      // converted weight tile (two halves)
  static constexpr int BUDGET = 216 * 1024 - W8_CBUF * C_BYTES;
  static constexpr int STAGES = BUDGET / STAGE_BYTES > 6 ? 6 : BUDGET / STAGE_BYTES;
  static constexpr uint32_t TMEM_COLS = tmem_cols_for(2 * BN);
};

// Two e4m3 (bytes sel_lo, sel_hi of w, selected by the byte_perm selector)
// -> bf16x2 holding value * 2^-120 exactly: sign to bit 15, exponent and
// mantissa bits shifted into the bf16 exponent/mantissa (e4m3 bias 7 vs
// bf16 bias 127; e4m3 subnormals land on bf16 subnormals).
__device__ __forceinline__ uint32_t e4m3x2_bits_to_bf16x2(uint32_t w, uint32_t sel) {
  const uint32_t t = __byte_perm(w, 0u, sel);
  return (t & 0x80008000u) | ((t >> 4) & 0x07F007F0u);
}

template <int BN>
__device__ __forceinline__ void w8_gemm_body(const CUtensorMap* tmW, const CUtensorMap* tmX,
                                             const float* __restrict__ w_scale, const int4* __restrict__ chunks,
                                             const int* __restrict__ meta, bf16* out, const bf16* residual, int O,
                                             int K, int ldo, int mode) {
  using C = W8Cfg<BN>;
  constexpr int STAGES = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sC = smem;                                  // [W8_CBUF][2 halves][128 rows x 128 B] bf16
  uint8_t* sA = sC + W8_CBUF * C::C_BYTES;             // [STAGES][128 x 128 B] e4m3
  uint8_t* sB = sA + STAGES * C::A8_BYTES;             // [STAGES][2 halves][BN x 128 B] bf16
  float* sws = reinterpret_cast<float*>(sB + STAGES * C::B_BYTES);  // [2][MAX_KB]
  uint64_t* full = reinterpret_cast<uint64_t*>(sws + 2 * MAX_KB);
  uint64_t* empty = full + STAGES;
  uint64_t* cfull = empty + STAGES;
  uint64_t* cempty = cfull + W8_CBUF;
  uint64_t* tfull = cempty + W8_CBUF;
  uint64_t* tempty = tfull + 2;
  uint64_t* sfull = tempty + 2;
  uint64_t* sempty = sfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sempty + 2);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int KB = K / QBLK;
  const int KBp = kb_pad(KB);
  const int num_ob = O / 128;
  const int num_chunks = meta[0];
  const int num_units = num_chunks * num_ob;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 5);  // 4 converter warps (A read) + the MMA commit (B read)
    }
    for (int c = 0; c < W8_CBUF; ++c) {
      mbar_init(&cfull[c], 4);
      mbar_init(&cempty[c], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 4);
      mbar_init(&sfull[a], 1);
      mbar_init(&sempty[a], 4);
    }
    *abort_flag = (KB > MAX_KB || (K % QBLK) || (O % 128)) ? 1 : 0;
    if (*abort_flag) set_status(FB_KERR_BAD_ARG);
    fence_barrier_init();
    fence_proxy_async();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(tmW);
    tma_prefetch_desc(tmX);
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
    // ---------------- producer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0, j = 0;
      const uint64_t pol = policy_evict_first();
      for (int u = blockIdx.x; u < num_units && !*(volatile int*)abort_flag; u += gridDim.x, ++j) {
        const int c = u % num_chunks, ob = u / num_chunks;
        const int4 ch = chunks[c];
        const int wrow = ch.x * O + ob * 128;
        const uint32_t slot = j & 1;
        if (!mbar_wait(&sempty[slot], ((j >> 1) & 1) ^ 1, FB_KERR_TIMEOUT_EMPTY)) {
          *(volatile int*)abort_flag = 1;
          break;
        }
        mbar_arrive_expect_tx(&sfull[slot], KBp * 4);
        bulk_load(sws + slot * MAX_KB, w_scale + (static_cast<size_t>(ch.x) * num_ob + ob) * KBp, KBp * 4,
                  &sfull[slot]);
        const int pf = pf_dist(mode);
        for (int kb = 0; kb < min(pf, KB); ++kb) tma_prefetch_2d(tmW, kb * QBLK, wrow);
        for (int kb = 0; kb < KB; ++kb) {
          if (pf && kb + pf < KB) tma_prefetch_2d(tmW, (kb + pf) * QBLK, wrow);
          if (!mbar_wait(&empty[stage], phase ^ 1, FB_KERR_TIMEOUT_EMPTY)) {
            *(volatile int*)abort_flag = 1;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
          if (mode & EPI_W_STREAM)
            tma_load_2d_hint(sA + stage * C::A8_BYTES, tmW, &full[stage], kb * QBLK, wrow, pol);
          else
            tma_load_2d(sA + stage * C::A8_BYTES, tmW, &full[stage], kb * QBLK, wrow);
          uint8_t* b = sB + stage * C::B_BYTES;
          tma_load_2d(b, tmX, &full[stage], kb * QBLK, ch.y);
          tma_load_2d(b + BN * 128, tmX, &full[stage], kb * QBLK + 64, ch.y);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      for (int s = 0; s < STAGES; ++s) {
        mbar_wait(&empty[stage], phase ^ 1, FB_KERR_TIMEOUT_EMPTY);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
      for (int s = 0; s < 2; ++s, ++j) mbar_wait(&sempty[j & 1], ((j >> 1) & 1) ^ 1, FB_KERR_TIMEOUT_EMPTY);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16<128, BN>();
      int stage = 0, cb = 0;
      uint32_t phase = 0, cphase = 0;
      int it = 0;
      for (int u = blockIdx.x; u < num_units && !*(volatile int*)abort_flag; u += gridDim.x, ++it) {
        const int acc = it & 1;
        if (!mbar_wait(&tempty[acc], ((it >> 1) & 1) ^ 1, FB_KERR_TIMEOUT_TMEM)) {
          *(volatile int*)abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        bool ok = true;
        for (int kb = 0; kb < KB; ++kb) {
          if (!mbar_wait(&full[stage], phase, FB_KERR_TIMEOUT_FULL)) {
            ok = false;
            break;
          }
          if (!mbar_wait(&cfull[cb], cphase, FB_KERR_TIMEOUT_FULL)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const uint64_t adesc = sdesc_sw128(smem_u32(sC + cb * C::C_BYTES + h * (C::C_BYTES / 2)));
            const uint64_t bdesc = sdesc_sw128(smem_u32(sB + stage * C::B_BYTES + h * BN * 128));
#pragma unroll
            for (int k = 0; k < 4; ++k)
              mma_bf16(d_tmem, adesc + (uint64_t)(k * 2), bdesc + (uint64_t)(k * 2), idesc,
                       (kb > 0 || h > 0 || k > 0) ? 1u : 0u);
          }
          mma_commit(&empty[stage]);
          mma_commit(&cempty[cb]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
          if (++cb == W8_CBUF) {
            cb = 0;
            cphase ^= 1;
          }
        }
        mma_commit(&tfull[acc]);
        if (!ok) {
          *(volatile int*)abort_flag = 1;
          break;
        }
      }
    }
  } else if (warp < 6) {
    // ---------------- converters: thread r dequantises weight row r ----------------
    const int r = threadIdx.x - 64;
    const int sw7 = r & 7;
    int stage = 0, cb = 0;
    uint32_t phase = 0, cphase = 0, j = 0;
    for (int u = blockIdx.x; u < num_units && !*(volatile int*)abort_flag; u += gridDim.x, ++j) {
      const uint32_t slot = j & 1;
      if (!mbar_wait(&sfull[slot], (j >> 1) & 1, FB_KERR_TIMEOUT_FULL)) {
        *(volatile int*)abort_flag = 1;
        break;
      }
      const float* wsu = sws + slot * MAX_KB;
      bool ok = true;
      for (int kb = 0; kb < KB; ++kb) {
        if (!mbar_wait(&full[stage], phase, FB_KERR_TIMEOUT_FULL) ||
            !mbar_wait(&cempty[cb], cphase ^ 1, FB_KERR_TIMEOUT_EMPTY)) {
          ok = false;
          break;
        }
        // bf16(sw * 2^120) times the exact bf16 image (value * 2^-120) of each e4m3
        const bf16 s = __float2bfloat16(wsu[kb] * 1.329227995784916e36f);
        const bf162 s2 = __halves2bfloat162(s, s);
        const uint8_t* arow = sA + stage * C::A8_BYTES + r * 128;
        uint8_t* crow = sC + cb * C::C_BYTES + r * 128;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const uint4 in = *reinterpret_cast<const uint4*>(arow + ((q ^ sw7) << 4));
          const uint32_t wv[4] = {in.x, in.y, in.z, in.w};
          uint32_t o[8];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            uint32_t lo = e4m3x2_bits_to_bf16x2(wv[i], 0x1404u);
            uint32_t hi = e4m3x2_bits_to_bf16x2(wv[i], 0x3424u);
            bf162 l2 = __hmul2(*reinterpret_cast<const bf162*>(&lo), s2);
            bf162 h2 = __hmul2(*reinterpret_cast<const bf162*>(&hi), s2);
            o[2 * i] = *reinterpret_cast<const uint32_t*>(&l2);
            o[2 * i + 1] = *reinterpret_cast<const uint32_t*>(&h2);
          }
          // fp8 chunk q = elements 16q..16q+15 -> bf16 chunks 2q, 2q+1 of half q / 4
          uint8_t* half = crow + (q >> 2) * (C::C_BYTES / 2);
          const int c0 = (2 * q) & 7;
          *reinterpret_cast<uint4*>(half + ((c0 ^ sw7) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
          *reinterpret_cast<uint4*>(half + (((c0 + 1) ^ sw7) << 4)) = make_uint4(o[4], o[5], o[6], o[7]);
        }
        fence_proxy_async();  // generic-proxy smem writes -> visible to the tensor core
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&cfull[cb]);
          mbar_arrive(&empty[stage]);
        }
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
        if (++cb == W8_CBUF) {
          cb = 0;
          cphase ^= 1;
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sempty[slot]);
      if (!ok) {
        *(volatile int*)abort_flag = 1;
        break;
      }
    }
  } else {
    // ---------------- epilogue (warps 6-9) ----------------
    const int quarter = warp & 3;
    int it = 0;
    for (int u = blockIdx.x; u < num_units && !*(volatile int*)abort_flag; u += gridDim.x, ++it) {
      const int c = u % num_chunks, ob = u / num_chunks;
      const int4 ch = chunks[c];
      const int acc = it & 1;
      if (!mbar_wait(&tfull[acc], (it >> 1) & 1, FB_KERR_TIMEOUT_TMEM)) {
        *(volatile int*)abort_flag = 1;
        break;
      }
      tc_fence_after();
      const int o = ob * 128 + quarter * 32 + lane;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * BN;
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 16) {
        uint32_t rr[16];
        tmem_ld16(t_row + c0, rr);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int t = c0 + i;
          if (t < ch.z) {
            const size_t idx = static_cast<size_t>(ch.y + t) * ldo + o;
            float v = __uint_as_float(rr[i]);
            if (mode & EPI_RESIDUAL) v += bf2f(residual[idx]);
            out[idx] = f2bf(v);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, C::TMEM_COLS);
}

}  // namespace

#define FB_W8_GEMM_INSTANCE(BN)                                                                                     \
  extern "C" __global__ void __launch_bounds__(W8_THREADS, 1) fb_moe_gemm_w8_bn##BN(                               \
      const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX, const float* w_scale,       \
      const int4* chunks, const int* meta, bf16* out, const bf16* residual, int O, int K, int ldo, int mode) {      \
    pdl_entry();                                                                                                    \
    w8_gemm_body<BN>(&tmW, &tmX, w_scale, chunks, meta, out, residual, O, K, ldo, mode);                           \
  }

FB_W8_GEMM_INSTANCE(32)
FB_W8_GEMM_INSTANCE(64)
FB_W8_GEMM_INSTANCE(128)

// Gather token rows into expert-sorted order: dst[pos[t * k + j]] = src[t]
// (bf16, H % 8 == 0). One CTA of 256 threads per token.
extern "C" __global__ void __launch_bounds__(256) fb_moe_scatter_rows(const bf16* __restrict__ src, int lds, int T,
                                                                     int H, const int* __restrict__ pos, int topk,
                                                                     bf16* __restrict__ dst) {
  pdl_entry();
  const int t = blockIdx.x;
  for (int c = threadIdx.x * 8; c < H; c += 256 * 8) {
    const uint4 v = *reinterpret_cast<const uint4*>(src + static_cast<size_t>(t) * lds + c);
    for (int j = 0; j < topk; ++j)
      *reinterpret_cast<uint4*>(dst + static_cast<size_t>(pos[t * topk + j]) * H + c) = v;
  }
}

// ==== expert parallelism: counts exchange, plan, fused quantise + dispatch ============
//
// Every rank owns experts [rank * El, (rank + 1) * El). Per MoE layer:
//   fb_ep_count     my pair count per global expert -> counts[rank][:] of every
//                   rank (P2P stores into symmetric memory); then a barrier
//   fb_ep_plan      from the full counts matrix: where each of my pairs lands in
//                   its owner's receive buffer (rows grouped by local expert,
//                   then source rank, then the source's pair order: a
//                   deterministic layout), and my own chunk table over the rows
//                   I will receive
//   fb_ep_dispatch  quantise each token once (e4m3, per-128 scales) and store
//                   its row + scales + (source rank, pair) into the owner's
//                   receive buffer over NVLink; then a barrier
// The expert GEMMs run on the receive buffer; the down projection's epilogue
// (EPI_PEER_COMBINE) writes each output row straight into the source rank's
// combine buffer; after a barrier fb_moe_combine_add_rmsnorm sums the k rows.

extern "C" __global__ void __launch_bounds__(256) fb_ep_count(const int* __restrict__ ids, int P, int E, int rank,
                                                             int world, unsigned long long base,
                                                             long long stride, long long counts_off) {
  pdl_entry();
  __shared__ int cnt[256];
  for (int e = threadIdx.x; e < E; e += 256) cnt[e] = 0;
  __syncthreads();
  for (int p = threadIdx.x; p < P; p += 256) atomicAdd(&cnt[ids[p]], 1);
  __syncthreads();
  for (int i = threadIdx.x; i < E * world; i += 256) {
    const int r = i / E, e = i % E;
    int* dst = reinterpret_cast<int*>(base + r * stride + counts_off);
    dst[rank * E + e] = cnt[e];
  }
}

// One CTA of 1024 threads. counts: [world][E] (this rank's copy).
extern "C" __global__ void __launch_bounds__(1024) fb_ep_plan(const int* __restrict__ counts,
                                                             const int* __restrict__ ids, int P, int E, int El,
                                                             int rank, int world, int bn, int* __restrict__ dst_row,
                                                             int4* __restrict__ chunks, int* __restrict__ meta) {
  pdl_entry();
  __shared__ int tot[256], base[256], before[256], run[256], coff[256];
  __shared__ int wcnt[32][256];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (E > 256) {
    if (tid == 0) set_status(FB_KERR_BAD_ARG);
    return;
  }
  for (int e = tid; e < E; e += 1024) {
    int t = 0, b = 0;
    for (int r = 0; r < world; ++r) {
      const int c = counts[r * E + e];
      t += c;
      if (r < rank) b += c;
    }
    tot[e] = t;
    before[e] = b;
    run[e] = 0;
  }
  __syncthreads();
  if (tid == 0) {
    // receive-side row base of every expert inside its owner's buffer, and
    // my chunk table over my local experts
    int nch = 0, rows = 0;
    for (int e = 0; e < E; ++e) {
      if (e % El == 0) rows = 0;
      base[e] = rows;
      rows += tot[e];
      if (e / El == rank) {
        coff[e] = nch;
        nch += (tot[e] + bn - 1) / bn;
      }
    }
    meta[0] = nch;
    int mine = 0;
    for (int le = 0; le < El; ++le) mine += tot[rank * El + le];
    meta[1] = mine;
  }
  __syncthreads();
  for (int le = tid; le < El; le += 1024) {
    const int e = rank * El + le, n = tot[e];
    for (int j = 0, r = 0; r < n; ++j, r += bn) chunks[coff[e] + j] = make_int4(le, base[e] + r, min(bn, n - r), 0);
  }
  for (int b0 = 0; b0 < P; b0 += 1024) {
    for (int i = tid; i < 32 * E; i += 1024) wcnt[i / E][i % E] = 0;
    __syncthreads();
    const int p = b0 + tid;
    const int e = p < P ? ids[p] : -1;
    const unsigned same = __match_any_sync(0xffffffffu, e);
    const int rk = __popc(same & ((1u << lane) - 1));
    if (e >= 0 && rk == 0) wcnt[warp][e] = __popc(same);
    __syncthreads();
    for (int x = tid; x < E; x += 1024) {
      int r0 = run[x];
      for (int w = 0; w < 32; ++w) {
        const int c = wcnt[w][x];
        wcnt[w][x] = r0;
        r0 += c;
      }
      run[x] = r0;
    }
    __syncthreads();
    if (e >= 0) dst_row[p] = base[e] + before[e] + wcnt[warp][e] + rk;
    __syncthreads();
  }
}

// Warp per (token, group of 4 scale blocks): quantise once, store to each of
// the token's k owners: e4m3 row, padded scale row and the row map entry.
extern "C" __global__ void __launch_bounds__(256) fb_ep_dispatch(
    const bf16* __restrict__ x, int ldx, int T, int H, const int* __restrict__ ids, const int* __restrict__ dst_row,
    int topk, int El, int rank, unsigned long long base, long long stride, long long q_off, long long s_off,
    long long map_off) {
  pdl_entry();
  constexpr int BPW = 4;
  const int nb = H / QBLK, nbp = kb_pad(nb);
  const int groups = (nb + BPW - 1) / BPW;
  const int w = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (w >= T * groups) return;
  const int t = w / groups, g = w % groups, b0 = g * BPW;
  uint32_t q[BPW];
  float sc[BPW];
#pragma unroll
  for (int i = 0; i < BPW; ++i) {
    const int b = b0 + i;
    if (b >= nb) break;
    const uint2 raw = *reinterpret_cast<const uint2*>(x + static_cast<size_t>(t) * ldx + b * QBLK + lane * 4);
    const float2 f0 = __bfloat1622float2(*reinterpret_cast<const bf162*>(&raw.x));
    const float2 f1 = __bfloat1622float2(*reinterpret_cast<const bf162*>(&raw.y));
    const float am = warp_max(fmaxf(fmaxf(fabsf(f0.x), fabsf(f0.y)), fmaxf(fabsf(f1.x), fabsf(f1.y))));
    const float s = fmaxf(am, 1e-12f) / FP8_MAX;
    const float inv = 1.f / s;
    q[i] = pack_e4m3x4(f0.x * inv, f0.y * inv, f1.x * inv, f1.y * inv);
    sc[i] = s;
  }
  for (int j = 0; j < topk; ++j) {
    const int pidx = t * topk + j;
    const int owner = ids[pidx] / El;
    const int row = dst_row[pidx];
    const unsigned long long win = base + owner * stride;
    uint32_t* dq = reinterpret_cast<uint32_t*>(win + q_off + static_cast<unsigned long long>(row) * H);
    float* ds = reinterpret_cast<float*>(win + s_off) + static_cast<size_t>(row) * nbp;
#pragma unroll
    for (int i = 0; i < BPW; ++i) {
      const int b = b0 + i;
      if (b >= nb) break;
      dq[b * 32 + lane] = q[i];
      if (lane == i) ds[b] = sc[i];
    }
    if (g == 0 && lane == 0) reinterpret_cast<int*>(win + map_off)[row] = (rank << 24) | pidx;
  }
}

// Block-scaled e4m3 [R, C] (scales [R/128, kb_pad(C/128)]) -> bf16 [R, C]:
// w = q * scale of its 128 x 128 block. One CTA per block, 8 elements per thread.
extern "C" __global__ void __launch_bounds__(256) fb_dequant_block_fp8(const uint8_t* __restrict__ q,
                                                                      const float* __restrict__ scales, int R,
                                                                      int Cc, bf16* __restrict__ out) {
  pdl_entry();
  const int bc = blockIdx.x, br = blockIdx.y;
  const float s = scales[static_cast<size_t>(br) * kb_pad(Cc / 128) + bc];
  const int r0 = threadIdx.x / 16, c0 = (threadIdx.x % 16) * 8;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const size_t row = static_cast<size_t>(br) * 128 + r0 + 16 * i;
    const uint2 raw = *reinterpret_cast<const uint2*>(q + row * Cc + bc * 128 + c0);
    const uint8_t* b = reinterpret_cast<const uint8_t*>(&raw);
    float f[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      __nv_fp8_e4m3 v;
      v.__x = b[j];
      f[j] = static_cast<float>(v) * s;
    }
    *reinterpret_cast<uint4*>(out + row * Cc + bc * 128 + c0) = pack8(f);
  }
}
