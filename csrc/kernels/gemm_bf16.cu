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
// Structure (one CTA per SM, persistent over work units):
//   warp 0      TMA producer: A/B tiles (128B-swizzled) into a STAGES-deep ring
//   warp 1      allocates TMEM; one elected lane issues tcgen05.mma (M=128,
//               N=BN, K=16) and tcgen05.commit to release smem stages and to
//               publish finished accumulators
//   warps 2-5   epilogue: tcgen05.ld (32 lanes x 16 columns, four per wait) ->
//               registers -> a shared-memory tile -> TMA store (transposed
//               decode outputs, residual tile loaded by TMA) or direct global
//               stores (prefill layout, multicast); when TMEM has room the
//               accumulators are double buffered so the epilogue of one unit
//               overlaps the next unit's MMAs
// A work unit is MT (1 or 2) 128-row A tiles x one BN-column B tile: with
// MT = 2 the B tile in shared memory feeds two MMAs per K step, halving the
// B bytes each SM has to pull per A byte (decode GEMMs are bound by how fast
// an SM can ingest tiles, and B is re-read for every A tile).
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
// mode bits 8..15: how many k-blocks ahead of the ring A tiles are prefetched into L2
constexpr int EPI_MCAST = 1 << 16;  // `out` is an NVLS multicast address: stores reach every rank
constexpr int EPI_TMA_OUT = 1 << 17;  // transposed output written by TMA stores through tmO (and tmR)
constexpr int EPI_A_CONST = 1 << 18;  // A is not written by any kernel of the step (weights): loaded before pdl_wait
// SwiGLU epilogue (MT == 2, swap-AB, TMA output): A is [gate; up] with M/2
// rows each; a unit's two A tiles are gate rows r..r+127 and the up rows of
// the same features (M/2 + r..), and the epilogue writes silu(gate) * up
// (bf16, [tokens][M/2]) instead of the two projections.
constexpr int EPI_SWIGLU = 1 << 19;
constexpr int NUM_THREADS = 192;

__device__ __forceinline__ void tma_store_2d(const void* tmap, const void* src, int32_t c0, int32_t c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                   reinterpret_cast<uint64_t>(tmap)),
               "r"(c0), "r"(c1), "r"(smem_u32(src))
               : "memory");
}
__device__ __forceinline__ void tma_store_3d(const void* tmap, const void* src, int32_t c0, int32_t c1, int32_t c2) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%1, %2, %3}], [%4];" ::"l"(
                   reinterpret_cast<uint64_t>(tmap)),
               "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(src))
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// At most one store group may still be reading shared memory.
__device__ __forceinline__ void bulk_wait_read_1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

constexpr uint32_t tmem_cols_for(int cols) {
  return cols <= 32 ? 32 : cols <= 64 ? 64 : cols <= 128 ? 128 : cols <= 256 ? 256 : 512;
}

// TMA-store epilogue of the transposed (swap-AB) output: per chunk of 32
// output columns (tokens) the epilogue threads convert their TMEM rows into a
// [32 tokens][128 features] tile in shared memory (bf16 output, or fp32 for a
// split-K slice) and one thread stores it with cp.async.bulk.tensor; two
// buffers alternate so the conversion of a chunk overlaps the store of the
// previous one. A residual tile comes in by TMA the same way. The epilogue
// threads then issue about one shared-memory store per output element and no
// global stores (the scalar-store epilogue left the last tile's stores on the
// critical path of every launch).
constexpr int EPI_COLS = 32;
constexpr int STG_BYTES = 2 * EPI_COLS * BM * 4;  // two fp32 buffers, or two bf16 + two residual buffers

template <int BN, int MT>
struct Cfg {
  static constexpr int A_BYTES = BM * BK * 2;         // one 128-row A tile per K step
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = MT * A_BYTES + B_BYTES;
  static constexpr int STAGES = (192 * 1024) / STAGE_BYTES > 8 ? 8 : (192 * 1024) / STAGE_BYTES;
  static constexpr int ACC_COLS = MT * BN;             // TMEM columns of one accumulator set
  static constexpr int ACC_BUFS = (2 * ACC_COLS <= 512) ? 2 : 1;
  static constexpr uint32_t TMEM_COLS = tmem_cols_for(ACC_BUFS * ACC_COLS);
};

// ---- fused all-reduce of a row-parallel (tensor-parallel) GEMM ----------------------
//
// fb_gemm_bf16_ar_bn{BN}: every rank computes its partial product of the same
// output and the epilogue all-reduces it tile by tile over NVSwitch while the
// next tile's MMAs run:
//   1. the partial tile is stored into P, this rank's slot of a symmetric
//      buffer (local memory bound to an NVLS multicast object);
//   2. one thread adds 1 to ready[tile] on every rank (multimem.red.release);
//   3. once ready[tile] == world here (all ranks' partials of the tile are
//      in place), the CTA reduces its 1/world share of the tile's rows in the
//      switch (multimem.ld_reduce, fp32 accumulation) and multicasts the sums
//      into O on every rank (multimem.st) - the reduce-scatter and the
//      all-gather of the tile - then adds 1 to done on every rank;
//   4. before exiting, every CTA waits for done == world * tiles here, so the
//      kernel's completion means O holds the full sum on this rank.
// Every rank runs the same tiles on the same CTAs in the same order, and a
// CTA signals its tile before it waits for anyone, so no CTA waits for work
// that cannot progress; all waits are bounded.
// Counters live in a control block per buffer in symmetric memory: an epoch
// word E (local, +1 by the last CTA to exit), a CTA exit ticket, done[2] and
// ready[2][AR_MAX_TILES], indexed by the parity of E. A launch clears the
// other parity's counters before it signals anything; every rank's next use
// of that parity comes after this launch has completed everywhere.
constexpr int EPI_AR = 1 << 20;
constexpr int AR_EPOCH = 0, AR_TICKET = 1, AR_DONE = 2, AR_READY = 16;
constexpr int AR_MAX_TILES = 4096;
struct ArArgs {
  uint64_t p_local;   // this rank's P (row stride ldo, bf16)
  uint64_t p_mc;      // P through the multicast object
  uint64_t o_mc;      // O (same layout as P) through the multicast object
  uint64_t flags;     // this rank's control block
  uint64_t flags_mc;  // the control block through the multicast object
  int rank, world;
};
__device__ __forceinline__ void mc_red_add_release(uint64_t addr, uint32_t v) {
  asm volatile("multimem.red.release.sys.global.add.u32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys_u32(uint64_t addr) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
  return v;
}
// Bounded wait until the local counter at addr reaches want (false on timeout).
__device__ __forceinline__ bool wait_counter(uint64_t addr, uint32_t want) {
  const uint64_t t0 = globaltimer();
  uint32_t spins = 0;
  while (static_cast<int32_t>(ld_acquire_sys_u32(addr) - want) < 0) {
    if ((++spins & 255u) == 0 && globaltimer() - t0 > FB_WAIT_NS) {
      set_status(FB_KERR_TIMEOUT_PEER);
      return false;
    }
  }
  return true;
}

template <int BN, int MT, bool AR = false>
__device__ __forceinline__ void gemm_body(const CUtensorMap* tmA, const CUtensorMap* tmB, const CUtensorMap* tmO,
                                          const CUtensorMap* tmR, bf16* __restrict__ out, const bf16* residual, int M,
                                          int N, int K, int ldo, int mode, int splits, float* __restrict__ ws,
                                          long long split_stride, ArArgs ar = ArArgs{}) {
  using C = Cfg<BN, MT>;
  constexpr int STAGES = C::STAGES;
  constexpr int NBUF = C::ACC_BUFS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;                               // [STAGES][MT][128 x 64]
  uint8_t* sB = smem + STAGES * MT * C::A_BYTES;     // [STAGES][BN x 64]
  uint8_t* stg = smem + STAGES * C::STAGE_BYTES;  // epilogue tiles (STG_BYTES)
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * C::STAGE_BYTES + STG_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* ebar = tempty + 2;  // the four epilogue warps' rendezvous (staging buffer hand-over)
  uint64_t* rbar = ebar + 1;    // residual tile loads, one per buffer
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(rbar + 2);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_m = (M + BM * MT - 1) / (BM * MT);   // units along M
  const int num_n = (N + BN - 1) / BN;
  const int KB = (K + BK - 1) / BK;
  const int kb_per = (KB + splits - 1) / splits;
  const int num_units = num_m * num_n * splits;
  // First A row of tile mt of unit row-block m_blk.
  auto a_row = [&](int m_blk, int mt) {
    return (mode & EPI_SWIGLU) ? mt * (M / 2) + m_blk * BM : (m_blk * MT + mt) * BM;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 4);
    }
    mbar_init(ebar, 4);
    mbar_init(&rbar[0], 1);
    mbar_init(&rbar[1], 1);
    *abort_flag = 0;
    fence_barrier_init();
    fence_proxy_async();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(tmA);
    tma_prefetch_desc(tmB);
    if (mode & EPI_TMA_OUT) {
      tma_prefetch_desc(tmO);
      if (mode & EPI_RESIDUAL) tma_prefetch_desc(tmR);
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_trigger();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      const uint64_t pol = policy_evict_first();
      const int pf_dist = (mode >> 8) & 0xFF;  // k-blocks of L2 prefetch lead (0 = off)
      auto load_a = [&](int st, int kb, int m_blk) {
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          uint8_t* dst = sA + (st * MT + mt) * C::A_BYTES;
          const int row = a_row(m_blk, mt);
          if (mode & EPI_A_STREAM)
            tma_load_2d_hint(dst, tmA, &full[st], kb * BK, row, pol);
          else
            tma_load_2d(dst, tmA, &full[st], kb * BK, row);
        }
      };
      // Before waiting for the previous kernel: the first unit's A tiles of
      // the whole ring, when A is an operand no kernel of the step writes
      // (the weights of a swap-AB GEMM; EPI_A_CONST). B (activations) and the
      // outputs wait for pdl_wait below.
      int pre = 0;
      if ((mode & EPI_A_CONST) && blockIdx.x < num_units) {
        const int mn = blockIdx.x / splits, sp = blockIdx.x % splits;
        const int kb0 = sp * kb_per, kb1 = min(KB, kb0 + kb_per);
        pre = min(STAGES, kb1 - kb0);
        for (int i = 0; i < pre; ++i) {
          mbar_arrive_expect_tx(&full[i], C::STAGE_BYTES);
          load_a(i, kb0 + i, mn % num_m);
        }
      }
      pdl_wait();
      for (int u = blockIdx.x; u < num_units && !*(volatile int*)abort_flag; u += gridDim.x) {
        const int mn = u / splits, sp = u % splits;
        const int m_blk = mn % num_m, n_blk = mn / num_m;
        const int kb0 = sp * kb_per, kb1 = min(KB, kb0 + kb_per);
        // Streamed A tiles: keep the L2 pf_dist k-blocks ahead of the ring.
        for (int kb = kb0; kb < min(kb1, kb0 + pf_dist); ++kb)
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) tma_prefetch_2d(tmA, kb * BK, a_row(m_blk, mt));
        for (int kb = kb0; kb < kb1; ++kb) {
          if (pf_dist && kb + pf_dist < kb1) {
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) tma_prefetch_2d(tmA, (kb + pf_dist) * BK, a_row(m_blk, mt));
          }
          if (pre > 0 && u == blockIdx.x && kb - kb0 < pre) {
            // stage armed and its A tiles issued before pdl_wait
          } else {
            if (!mbar_wait(&empty[stage], phase ^ 1, FB_KERR_TIMEOUT_EMPTY)) {
              *(volatile int*)abort_flag = 1;
              break;
            }
            mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
            // Operands read exactly once per launch (decode weights) are hinted
            // evict-first so they do not push reused activations out of L2.
            load_a(stage, kb, m_blk);
          }
          if (mode & EPI_B_STREAM)
            tma_load_2d_hint(sB + stage * C::B_BYTES, tmB, &full[stage], kb * BK, n_blk * BN, pol);
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
      for (int u = blockIdx.x; u < num_units && !*(volatile int*)abort_flag; u += gridDim.x, ++it) {
        const int sp = u % splits;
        const int kb0 = sp * kb_per, kb1 = min(KB, kb0 + kb_per);
        const int acc = NBUF == 2 ? (it & 1) : 0;
        const uint32_t aphase = NBUF == 2 ? ((it >> 1) & 1) : (it & 1);
        if (!mbar_wait(&tempty[acc], aphase ^ 1, FB_KERR_TIMEOUT_TMEM)) {
          *(volatile int*)abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * C::ACC_COLS;
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, FB_KERR_TIMEOUT_FULL)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t bdesc = sdesc_sw128(smem_u32(sB + stage * C::B_BYTES));
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) {
            const uint64_t adesc = sdesc_sw128(smem_u32(sA + (stage * MT + mt) * C::A_BYTES));
#pragma unroll
            for (int k = 0; k < BK / 16; ++k) {
              // +32 bytes per 16-element K step inside the 128-byte swizzle row.
              mma_bf16(d_tmem + mt * BN, adesc + (uint64_t)(k * 2), bdesc + (uint64_t)(k * 2), idesc,
                       (kb > kb0 || k > 0) ? 1u : 0u);
            }
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
    pdl_wait();  // residual reads and output writes follow the previous kernel
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    const int et = threadIdx.x - 64;  // 0..127 over the four epilogue warps; 0 issues the tile stores
    const bool tma_out = (mode & EPI_TMA_OUT) && (mode & EPI_TRANSPOSE) && !(mode & EPI_MCAST);
    uint32_t ephase = 0, rphase = 0;  // rphase bit b: parity of residual buffer b
    uint32_t chunk = 0;  // epilogue chunks so far: buffer = chunk & 1
    bool ok = true;
    // Bounded rendezvous of the four epilogue warps: a warp that gave up on a
    // wait never leaves the others blocked.
    auto epi_sync = [&]() -> bool {
      __syncwarp();
      if (lane == 0) mbar_arrive(ebar);
      const bool done = mbar_wait(ebar, ephase, FB_KERR_TIMEOUT_TMEM);
      ephase ^= 1;
      return done;
    };
    uint32_t ar_par = 0;  // parity of this launch's counters
    if constexpr (AR) {
      uint32_t* fl = reinterpret_cast<uint32_t*>(ar.flags);
      const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(fl + AR_EPOCH);
      ar_par = epoch & 1u;
      // Clear the other parity (this CTA's share) before signalling anything.
      uint32_t* old_ready = fl + AR_READY + (ar_par ^ 1u) * AR_MAX_TILES;
      for (int i = blockIdx.x * 128 + et; i < AR_MAX_TILES; i += gridDim.x * 128) old_ready[i] = 0;
      if (blockIdx.x == 0 && et == 0) fl[AR_DONE + (ar_par ^ 1u)] = 0;
      __threadfence_system();
    }
    int it = 0;
    for (int u = blockIdx.x; ok && u < num_units && !*(volatile int*)abort_flag; u += gridDim.x, ++it) {
      const int mn = u / splits, sp = u % splits;
      const int m_blk = mn % num_m, n_blk = mn / num_m;
      const int acc = NBUF == 2 ? (it & 1) : 0;
      const uint32_t aphase = NBUF == 2 ? ((it >> 1) & 1) : (it & 1);
      if (!mbar_wait(&tfull[acc], aphase, FB_KERR_TIMEOUT_TMEM)) {
        *(volatile int*)abort_flag = 1;
        break;
      }
      tc_fence_after();
      float* part = splits > 1 ? ws + static_cast<size_t>(sp) * split_stride : nullptr;
      if (MT == 2 && (mode & EPI_SWIGLU) && tma_out) {
        // act[token][feature] = silu(gate) * up: this thread holds both
        // projections of feature m_blk * 128 + f (accumulators 0 and 1).
        constexpr int EC = BN < EPI_COLS ? BN : EPI_COLS;
        const int f = quarter * 32 + lane;
        const uint32_t t_g = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * C::ACC_COLS;
#pragma unroll 1
        for (int c1 = 0; c1 < BN && ok; c1 += EC, ++chunk) {
          const int buf = chunk & 1;
          bf16* sb = reinterpret_cast<bf16*>(stg) + buf * (EPI_COLS * BM);
          uint32_t rg[EC], ru[EC];
#pragma unroll
          for (int j = 0; j < EC / 16; ++j) {
            tmem_ld16(t_g + c1 + 16 * j, *reinterpret_cast<uint32_t(*)[16]>(rg + 16 * j));
            tmem_ld16(t_g + BN + c1 + 16 * j, *reinterpret_cast<uint32_t(*)[16]>(ru + 16 * j));
          }
          tmem_ld_wait();
          if (et == 0 && chunk >= 2) bulk_wait_read_1();  // this buffer's previous store has read it
          if (!(ok = epi_sync())) break;
#pragma unroll
          for (int t = 0; t < EC; ++t) {
            const float g = __uint_as_float(rg[t]);
            sb[t * BM + f] = f2bf(g / (1.f + __expf(-g)) * __uint_as_float(ru[t]));
          }
          fence_proxy_async();
          if (!(ok = epi_sync())) break;
          if (et == 0) {
            tma_store_2d(tmO, sb, m_blk * BM, n_blk * BN + c1);
            bulk_commit();
          }
        }
      } else
#pragma unroll 1
      for (int mt = 0; mt < MT && ok; ++mt) {
        const int gm = (m_blk * MT + mt) * BM + quarter * 32 + lane;  // D row of this thread
        const uint32_t t_row =
            tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * C::ACC_COLS + mt * BN;
        // 64 columns (four 16-column TMEM loads) per wait: one TMEM round trip
        // per 64 columns instead of per 16.
        if (tma_out) {
          constexpr int EC = BN < EPI_COLS ? BN : EPI_COLS;
          const int gm0 = (m_blk * MT + mt) * BM;
          const int f = quarter * 32 + lane;  // feature (row of D) this thread holds
#pragma unroll 1
          for (int c1 = 0; c1 < BN && ok; c1 += EC, ++chunk) {
            const int buf = chunk & 1;
            const int gn0 = n_blk * BN + c1;
            float* sf = reinterpret_cast<float*>(stg) + buf * (EPI_COLS * BM);          // fp32 tile
            bf16* sb = reinterpret_cast<bf16*>(stg) + buf * (EPI_COLS * BM);            // bf16 tile
            bf16* sr = reinterpret_cast<bf16*>(stg + STG_BYTES / 2) + buf * (EPI_COLS * BM);  // residual
            uint32_t rr[EC];
#pragma unroll
            for (int j = 0; j < EC / 16; ++j)
              tmem_ld16(t_row + c1 + 16 * j, *reinterpret_cast<uint32_t(*)[16]>(rr + 16 * j));
            tmem_ld_wait();
            if (et == 0 && chunk >= 2) bulk_wait_read_1();  // this buffer's previous store has read it
            if (!(ok = epi_sync())) break;
            if (!part && (mode & EPI_RESIDUAL)) {
              if (et == 0) {
                mbar_arrive_expect_tx(&rbar[buf], EC * BM * 2);
                tma_load_2d(sr, tmR, &rbar[buf], gm0, gn0);
              }
              if (!(ok = mbar_wait(&rbar[buf], (rphase >> buf) & 1u, FB_KERR_TIMEOUT_FULL))) break;
              rphase ^= 1u << buf;
            }
            if (part) {
#pragma unroll
              for (int t = 0; t < EC; ++t) sf[t * BM + f] = __uint_as_float(rr[t]);
            } else if (mode & EPI_RESIDUAL) {
#pragma unroll
              for (int t = 0; t < EC; ++t) sb[t * BM + f] = f2bf(__uint_as_float(rr[t]) + bf2f(sr[t * BM + f]));
            } else {
#pragma unroll
              for (int t = 0; t < EC; ++t) sb[t * BM + f] = f2bf(__uint_as_float(rr[t]));
            }
            fence_proxy_async();  // generic-proxy writes -> visible to the TMA engine
            if (!(ok = epi_sync())) break;
            if (et == 0) {
              if (part)
                tma_store_3d(tmO, sf, gm0, gn0, sp);
              else
                tma_store_2d(tmO, sb, gm0, gn0);
              bulk_commit();
            }
          }
          continue;
        }
        constexpr int CH = BN < 64 ? BN : 64;
#pragma unroll 1
        for (int c1 = 0; c1 < BN; c1 += CH) {
          uint32_t rr[CH];
#pragma unroll
          for (int j = 0; j < CH / 16; ++j)
            tmem_ld16(t_row + c1 + 16 * j, *reinterpret_cast<uint32_t(*)[16]>(rr + 16 * j));
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < CH / 16; ++j) {
          const uint32_t* r = rr + 16 * j;
          const int c0 = c1 + 16 * j;
          const int gn0 = n_blk * BN + c0;
          if ((mode & EPI_MCAST) && (mode & EPI_TRANSPOSE)) {
            // Multicast store of bf16 pairs: lanes hold consecutive output
            // features; even lanes store (own, neighbour) as one bf16x2.
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const float mine = __uint_as_float(r[i]);
              const float nb = __shfl_xor_sync(0xffffffffu, mine, 1);
              const int gn = gn0 + i;
              if (!(lane & 1) && gm < M && gn < N) {
                const bf162 pr = __floats2bfloat162_rn(mine, nb);
                const uint64_t dst = reinterpret_cast<uint64_t>(out) + (static_cast<uint64_t>(gn) * ldo + gm) * 2;
                asm volatile("multimem.st.relaxed.sys.global.bf16x2 [%0], %1;" ::"l"(dst),
                             "r"(*reinterpret_cast<const uint32_t*>(&pr))
                             : "memory");
              }
            }
            continue;
          }
          if (gm >= M) continue;
          if (mode & EPI_MCAST) {
            // Row-major multicast store: 16 consecutive columns = 2 x 16 B.
            if (gn0 + 16 <= N) {
              float f[16];
#pragma unroll
              for (int i = 0; i < 16; ++i) f[i] = __uint_as_float(r[i]);
              uint32_t u[8];
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                const bf162 pr = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
                u[i] = *reinterpret_cast<const uint32_t*>(&pr);
              }
              const uint64_t dst = reinterpret_cast<uint64_t>(out) + (static_cast<uint64_t>(gm) * ldo + gn0) * 2;
              asm volatile("multimem.st.relaxed.sys.global.v4.bf16x2 [%0], {%1,%2,%3,%4};" ::"l"(dst), "r"(u[0]),
                           "r"(u[1]), "r"(u[2]), "r"(u[3])
                           : "memory");
              asm volatile("multimem.st.relaxed.sys.global.v4.bf16x2 [%0], {%1,%2,%3,%4};" ::"l"(dst + 16),
                           "r"(u[4]), "r"(u[5]), "r"(u[6]), "r"(u[7])
                           : "memory");
            }
            continue;
          }
          if (part) {
            // Split-K: fp32 slice in the output's layout.
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
          } else if (mode & EPI_TRANSPOSE) {
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
              float lo[8], hi[8];
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                lo[i] = __uint_as_float(r[i]);
                hi[i] = __uint_as_float(r[8 + i]);
              }
              if (mode & EPI_RESIDUAL) {
                float a[8], b[8];
                unpack8(*reinterpret_cast<const uint4*>(residual + base), a);
                unpack8(*reinterpret_cast<const uint4*>(residual + base + 8), b);
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                  lo[i] += a[i];
                  hi[i] += b[i];
                }
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
      }
      if (!ok) {
        *(volatile int*)abort_flag = 1;
        break;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      if constexpr (AR) {
        // (1) this rank's partial tile is complete in P and visible system-wide
        if (et == 0 && tma_out) {
          bulk_wait_all();
          asm volatile("fence.proxy.async.global;" ::: "memory");
        }
        __threadfence_system();
        if (!(ok = epi_sync())) break;
        // (2) announce it on every rank
        const uint64_t ready = AR_READY * 4ull + (ar_par * AR_MAX_TILES + u) * 4ull;
        if (et == 0) mc_red_add_release(ar.flags_mc + ready, 1);
        // (3) all ranks' partials of this tile are in P: reduce this rank's
        // share of its rows in the switch and multicast the sums into O
        if (et == 0 && !wait_counter(ar.flags + ready, static_cast<uint32_t>(ar.world)))
          *(volatile int*)abort_flag = 1;  // a peer never announced its tile: every thread stops
        if (!(ok = epi_sync()) || *(volatile int*)abort_flag) {
          ok = false;
          break;
        }
        (void)ld_acquire_sys_u32(ar.flags + ready);  // acquire for this thread's reads below
        const bool tr = (mode & EPI_TRANSPOSE) != 0;  // rows = tokens along N (swap-AB) or along M
        const int r0 = tr ? n_blk * BN : m_blk * BM, c0 = tr ? m_blk * BM : n_blk * BN;
        const int nr = min(tr ? BN : BM, (tr ? N : M) - r0), nc = min(tr ? BM : BN, (tr ? M : N) - c0);
        const int vpr = nc >> 3;  // 16-byte vectors per row (nc % 8 == 0: checked by the host)
        const int mine = (nr - ar.rank + ar.world - 1) / ar.world;  // rows r0 + rank + k * world
        const int nv = mine * vpr;
        constexpr int UNR = 8;
#pragma unroll 1
        for (int v0 = et; v0 < nv; v0 += 128 * UNR) {
          uint32_t q[UNR][4];
          uint64_t off[UNR];
#pragma unroll
          for (int j = 0; j < UNR; ++j) {
            const int v = v0 + j * 128;
            if (v < nv) {
              const int row = r0 + ar.rank + (v / vpr) * ar.world, col = c0 + (v % vpr) * 8;
              off[j] = (static_cast<uint64_t>(row) * ldo + col) * 2ull;
              asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0,%1,%2,%3}, [%4];"
                           : "=r"(q[j][0]), "=r"(q[j][1]), "=r"(q[j][2]), "=r"(q[j][3])
                           : "l"(ar.p_mc + off[j])
                           : "memory");
            }
          }
#pragma unroll
          for (int j = 0; j < UNR; ++j) {
            if (v0 + j * 128 < nv)
              asm volatile("multimem.st.relaxed.sys.global.v4.bf16x2 [%0], {%1,%2,%3,%4};" ::"l"(ar.o_mc + off[j]),
                           "r"(q[j][0]), "r"(q[j][1]), "r"(q[j][2]), "r"(q[j][3])
                           : "memory");
          }
        }
        __threadfence_system();
        if (!(ok = epi_sync())) break;
        if (et == 0) mc_red_add_release(ar.flags_mc + (AR_DONE + ar_par) * 4ull, 1);
      }
    }
    if (et == 0 && tma_out) bulk_wait_all();  // the tile stores have read shared memory and landed
    if constexpr (AR) {
      if (et == 0) {
        // (4) every rank's share of every tile has reached this rank's O
        if (ok) ok = wait_counter(ar.flags + (AR_DONE + ar_par) * 4ull,
                                  static_cast<uint32_t>(ar.world) * static_cast<uint32_t>(num_units));
        uint32_t* fl = reinterpret_cast<uint32_t*>(ar.flags);
        if (atomicAdd(fl + AR_TICKET, 1u) == gridDim.x - 1) {  // last CTA out: next launch, other parity
          fl[AR_TICKET] = 0;
          fl[AR_EPOCH] = fl[AR_EPOCH] + 1;
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

#define FB_GEMM_INSTANCE(BN, MT)                                                                                    \
  extern "C" __global__ void __launch_bounds__(NUM_THREADS, 1) fb_gemm_bf16_bn##BN##_m##MT(                         \
      const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,                             \
      const __grid_constant__ CUtensorMap tmO, const __grid_constant__ CUtensorMap tmR, bf16* out,                  \
      const bf16* residual, int M, int N, int K, int ldo, int mode, int splits, float* ws,                          \
      long long split_stride) {                                                                                      \
    gemm_body<BN, MT>(&tmA, &tmB, &tmO, &tmR, out, residual, M, N, K, ldo, mode, splits, ws, split_stride);        \
  }

#define FB_GEMM_AR_INSTANCE(BN)                                                                                     \
  extern "C" __global__ void __launch_bounds__(NUM_THREADS, 1) fb_gemm_bf16_ar_bn##BN(                              \
      const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,                             \
      const __grid_constant__ CUtensorMap tmO, bf16* out, int M, int N, int K, int ldo, int mode,                   \
      unsigned long long p_mc, unsigned long long o_mc, unsigned long long flags, unsigned long long flags_mc,        \
      int rank, int world) {                                                                                         \
    const ArArgs ar{reinterpret_cast<uint64_t>(out), p_mc, o_mc, flags, flags_mc, rank, world};                     \
    gemm_body<BN, 1, true>(&tmA, &tmB, &tmO, &tmO, out, nullptr, M, N, K, ldo, mode | EPI_AR, 1, nullptr, 0, ar);   \
  }

FB_GEMM_INSTANCE(16, 1)
FB_GEMM_INSTANCE(32, 1)
FB_GEMM_INSTANCE(64, 1)
FB_GEMM_INSTANCE(128, 1)
FB_GEMM_INSTANCE(256, 1)
FB_GEMM_INSTANCE(16, 2)
FB_GEMM_INSTANCE(32, 2)
FB_GEMM_INSTANCE(64, 2)
FB_GEMM_INSTANCE(128, 2)
FB_GEMM_INSTANCE(256, 2)
FB_GEMM_AR_INSTANCE(16)
FB_GEMM_AR_INSTANCE(32)
FB_GEMM_AR_INSTANCE(64)
FB_GEMM_AR_INSTANCE(128)
FB_GEMM_AR_INSTANCE(256)

// ==== stream-K variant (swap-AB decode GEMMs with more tiles than SMs) =================
//
// fb_gemm_sk_bn{BN}: the same TMA -> tcgen05 -> TMEM pipeline, but every CTA
// gets an equal share of the (tile, k-block) iterations instead of whole
// tiles, so 224 tiles on 148 SMs take 1.51 tile-times instead of 2. A CTA's
// range is cut into segments at tile boundaries; with at least one tile per
// CTA a tile is split between at most two neighbouring CTAs (b, b + 1). Both
// halves meet through slot b of a workspace: an atomic ticket (one per slot,
// taken by one epilogue thread for the whole 128-row tile) decides who
// arrives first; the first writes its fp32 partial and releases a flag, the
// second adds the partner's partial to its own (a + b == b + a in fp32, so
// the result does not depend on the order), stores the bf16 tile and resets
// the ticket and flag for the next launch. Nobody waits for a CTA that has
// not started: the first arriver never waits and the second only waits for a
// write already in progress (bounded).
// Output: transposed (out[token][feature]) with optional residual, through
// the same staged TMA-store epilogue as fb_gemm_bf16 (tmO / tmR required).
namespace {

__device__ __forceinline__ void st_release_gpu(int* p, int v) {
  asm volatile("st.release.gpu.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

template <int BN>
__device__ __forceinline__ void gemm_sk_body(const CUtensorMap* tmA, const CUtensorMap* tmB, const CUtensorMap* tmO,
                                             const CUtensorMap* tmR, int M, int N, int K, int mode,
                                             float* __restrict__ ws, int* __restrict__ flags) {
  using C = Cfg<BN, 1>;
  constexpr int STAGES = C::STAGES;
  constexpr int NBUF = C::ACC_BUFS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * C::A_BYTES;
  uint8_t* stg = smem + STAGES * C::STAGE_BYTES;  // epilogue tiles (STG_BYTES)
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * C::STAGE_BYTES + STG_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* ebar = tempty + 2;  // the four epilogue warps' rendezvous
  uint64_t* rbar = ebar + 1;    // residual tile loads, one per buffer
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(rbar + 2);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
  int* tile_ticket = abort_flag + 1;  // the ticket this CTA drew for its current split tile

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_m = (M + BM - 1) / BM;
  const int num_n = (N + BN - 1) / BN;
  const int KB = (K + BK - 1) / BK;
  const long long total = static_cast<long long>(num_m) * num_n * KB;
  const long long it0 = total * blockIdx.x / gridDim.x;
  const long long it1 = total * (blockIdx.x + 1) / gridDim.x;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 4);
    }
    mbar_init(ebar, 4);
    mbar_init(&rbar[0], 1);
    mbar_init(&rbar[1], 1);
    *abort_flag = 0;
    fence_barrier_init();
    fence_proxy_async();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(tmA);
    tma_prefetch_desc(tmB);
    tma_prefetch_desc(tmO);
    if (mode & EPI_RESIDUAL) tma_prefetch_desc(tmR);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_trigger();
  pdl_wait();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      const uint64_t pol = policy_evict_first();
      const int pf_dist = (mode >> 8) & 0xFF;
      for (long long it = it0; it < it1 && !*(volatile int*)abort_flag;) {
        const int tile = static_cast<int>(it / KB);
        const int kb0 = static_cast<int>(it % KB);
        const int kb1 = static_cast<int>(min(static_cast<long long>(KB), kb0 + (it1 - it)));
        const int m_blk = tile % num_m, n_blk = tile / num_m;
        for (int kb = kb0; kb < min(kb1, kb0 + pf_dist); ++kb) tma_prefetch_2d(tmA, kb * BK, m_blk * BM);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (pf_dist && kb + pf_dist < kb1) tma_prefetch_2d(tmA, (kb + pf_dist) * BK, m_blk * BM);
          if (!mbar_wait(&empty[stage], phase ^ 1, FB_KERR_TIMEOUT_EMPTY)) {
            *(volatile int*)abort_flag = 1;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
          if (mode & EPI_A_STREAM)
            tma_load_2d_hint(sA + stage * C::A_BYTES, tmA, &full[stage], kb * BK, m_blk * BM, pol);
          else
            tma_load_2d(sA + stage * C::A_BYTES, tmA, &full[stage], kb * BK, m_blk * BM);
          tma_load_2d(sB + stage * C::B_BYTES, tmB, &full[stage], kb * BK, n_blk * BN);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        it += kb1 - kb0;
      }
      for (int s = 0; s < STAGES; ++s) {
        mbar_wait(&empty[stage], phase ^ 1, FB_KERR_TIMEOUT_EMPTY);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer: one accumulator per segment ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16<BM, BN>();
      int stage = 0;
      uint32_t phase = 0;
      int seg = 0;
      for (long long it = it0; it < it1 && !*(volatile int*)abort_flag; ++seg) {
        const int kb0 = static_cast<int>(it % KB);
        const int kb1 = static_cast<int>(min(static_cast<long long>(KB), kb0 + (it1 - it)));
        const int acc = NBUF == 2 ? (seg & 1) : 0;
        const uint32_t aphase = NBUF == 2 ? ((seg >> 1) & 1) : (seg & 1);
        if (!mbar_wait(&tempty[acc], aphase ^ 1, FB_KERR_TIMEOUT_TMEM)) {
          *(volatile int*)abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * C::ACC_COLS;
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
          for (int k = 0; k < BK / 16; ++k)
            mma_bf16(d_tmem, adesc + (uint64_t)(k * 2), bdesc + (uint64_t)(k * 2), idesc,
                     (kb > kb0 || k > 0) ? 1u : 0u);
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
        it += kb1 - kb0;
      }
    }
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    constexpr int EC = BN < EPI_COLS ? BN : EPI_COLS;
    const int quarter = warp & 3;
    const int et = threadIdx.x - 64;    // 0..127; 0 draws tickets and issues the tile stores
    const int f = quarter * 32 + lane;  // D row (output feature within the tile) of this thread
    uint32_t ephase = 0, rphase = 0, chunk = 0;
    bool ok = true;
    auto epi_sync = [&]() -> bool {
      __syncwarp();
      if (lane == 0) mbar_arrive(ebar);
      const bool done = mbar_wait(ebar, ephase, FB_KERR_TIMEOUT_TMEM);
      ephase ^= 1;
      return done;
    };
    int seg = 0;
    for (long long it = it0; ok && it < it1 && !*(volatile int*)abort_flag; ++seg) {
      const int tile = static_cast<int>(it / KB);
      const int kb0 = static_cast<int>(it % KB);
      const int kb1 = static_cast<int>(min(static_cast<long long>(KB), kb0 + (it1 - it)));
      it += kb1 - kb0;
      const int m_blk = tile % num_m, n_blk = tile / num_m;
      const int acc = NBUF == 2 ? (seg & 1) : 0;
      const uint32_t aphase = NBUF == 2 ? ((seg >> 1) & 1) : (seg & 1);
      if (!mbar_wait(&tfull[acc], aphase, FB_KERR_TIMEOUT_TMEM)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int gm0 = m_blk * BM;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * C::ACC_COLS;
      // Split tile: the prefix owner is the CTA whose range ends inside it.
      const bool split = !(kb0 == 0 && kb1 == KB);
      const int slot = (kb0 == 0) ? blockIdx.x : blockIdx.x - 1;
      int* ticket = flags + slot * 8;
      int* ready = flags + slot * 8 + 4;
      float* part = ws + (static_cast<size_t>(slot) * BM + f) * BN;  // this thread's fp32 row
      bool first = false;
      if (split) {
        if (et == 0) *tile_ticket = atomicAdd(ticket, 1);
        if (!(ok = epi_sync())) break;
        first = *(volatile int*)tile_ticket == 0;
        if (!first) {
          // the partner is writing its partial: bounded wait for its flag
          const uint64_t t0 = globaltimer();
          uint32_t spins = 0;
          while (ld_acquire_gpu(ready) == 0) {
            if ((++spins & 255u) == 0 && globaltimer() - t0 > FB_WAIT_NS) {
              set_status(FB_KERR_TIMEOUT_PEER);
              ok = false;
              break;
            }
          }
          if (!ok) break;
        }
      }
      if (split && first) {
        // fp32 partial: row f of the slot, BN contiguous floats per thread
#pragma unroll 1
        for (int c1 = 0; c1 < BN; c1 += EC) {
          uint32_t rr[EC];
#pragma unroll
          for (int j = 0; j < EC / 16; ++j)
            tmem_ld16(t_row + c1 + 16 * j, *reinterpret_cast<uint32_t(*)[16]>(rr + 16 * j));
          tmem_ld_wait();
          float4* dst = reinterpret_cast<float4*>(part + c1);
#pragma unroll
          for (int i = 0; i < EC / 4; ++i)
            dst[i] = make_float4(__uint_as_float(rr[4 * i]), __uint_as_float(rr[4 * i + 1]),
                                 __uint_as_float(rr[4 * i + 2]), __uint_as_float(rr[4 * i + 3]));
        }
        __threadfence();
        if (!(ok = epi_sync())) break;  // all 128 rows written
        if (et == 0) st_release_gpu(ready, 1);
      } else {
        // whole tile, or the second half of a split one: bf16 [EC tokens][128
        // features] staging tiles stored by TMA, double-buffered
#pragma unroll 1
        for (int c1 = 0; c1 < BN && ok; c1 += EC, ++chunk) {
          const int buf = chunk & 1;
          const int gn0 = n_blk * BN + c1;
          bf16* sb = reinterpret_cast<bf16*>(stg) + buf * (EPI_COLS * BM);
          bf16* sr = reinterpret_cast<bf16*>(stg + STG_BYTES / 2) + buf * (EPI_COLS * BM);
          uint32_t rr[EC];
#pragma unroll
          for (int j = 0; j < EC / 16; ++j)
            tmem_ld16(t_row + c1 + 16 * j, *reinterpret_cast<uint32_t(*)[16]>(rr + 16 * j));
          tmem_ld_wait();
          float v[EC];
#pragma unroll
          for (int t = 0; t < EC; ++t) v[t] = __uint_as_float(rr[t]);
          if (split) {
#pragma unroll
            for (int i = 0; i < EC / 4; ++i) {
              const float4 q = __ldcg(reinterpret_cast<const float4*>(part + c1) + i);
              v[4 * i] += q.x;
              v[4 * i + 1] += q.y;
              v[4 * i + 2] += q.z;
              v[4 * i + 3] += q.w;
            }
          }
          if (et == 0 && chunk >= 2) bulk_wait_read_1();  // this buffer's previous store has read it
          if (!(ok = epi_sync())) break;
          if (mode & EPI_RESIDUAL) {
            if (et == 0) {
              mbar_arrive_expect_tx(&rbar[buf], EC * BM * 2);
              tma_load_2d(sr, tmR, &rbar[buf], gm0, gn0);
            }
            if (!(ok = mbar_wait(&rbar[buf], (rphase >> buf) & 1u, FB_KERR_TIMEOUT_FULL))) break;
            rphase ^= 1u << buf;
#pragma unroll
            for (int t = 0; t < EC; ++t) sb[t * BM + f] = f2bf(v[t] + bf2f(sr[t * BM + f]));
          } else {
#pragma unroll
            for (int t = 0; t < EC; ++t) sb[t * BM + f] = f2bf(v[t]);
          }
          fence_proxy_async();  // generic-proxy writes -> visible to the TMA engine
          if (!(ok = epi_sync())) break;
          if (et == 0) {
            tma_store_2d(tmO, sb, gm0, gn0);
            bulk_commit();
          }
        }
        // every thread read its partner rows before the last rendezvous
        if (ok && split && et == 0) {
          *ticket = 0;  // reset for the next launch (kernel boundary orders it)
          *ready = 0;
        }
      }
      if (!ok) break;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
    if (!ok) *(volatile int*)abort_flag = 1;
    if (et == 0) bulk_wait_all();  // the tile stores have read shared memory and landed
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, C::TMEM_COLS);
}

}  // namespace

#define FB_GEMM_SK_INSTANCE(BN)                                                                                     \
  extern "C" __global__ void __launch_bounds__(NUM_THREADS, 1) fb_gemm_sk_bn##BN(                                  \
      const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,                             \
      const __grid_constant__ CUtensorMap tmO, const __grid_constant__ CUtensorMap tmR, int M, int N, int K,        \
      int mode, float* ws, int* flags) {                                                                            \
    gemm_sk_body<BN>(&tmA, &tmB, &tmO, &tmR, M, N, K, mode, ws, flags);                                             \
  }

FB_GEMM_SK_INSTANCE(16)
FB_GEMM_SK_INSTANCE(32)
FB_GEMM_SK_INSTANCE(64)
FB_GEMM_SK_INSTANCE(128)
FB_GEMM_SK_INSTANCE(256)

// ==== fused gate/up + SwiGLU, stream-K over every SM ====================================
//
// fb_gemm_swiglu_sk_bn256: the decode-step gate/up projection of
// fb_gemm_bf16_bn256_m2 (units of 128 features: gate rows f.., up rows
// I + f..; both accumulators in TMEM; epilogue silu(gate) * up) with the
// (unit, k-block) iterations shared equally by all CTAs. With fewer units
// than SMs (Llama-3-8B: 112 units on 148 SMs) the one-unit-per-CTA kernel
// leaves SMs idle; here CTA b runs iterations [T*b/G, T*(b+1)/G) of the
// T = units * k-blocks, so a unit is cut into pieces run by consecutive CTAs
// (at most SWIGLU_SK_MAXP; the host checks). A piece's CTA draws a ticket for
// its unit when its MMAs are done; every piece but the last to draw writes
// its fp32 gate and up rows to its slot of `ws` and raises its ready flag;
// the last waits for the others' flags (bounded), sums the pieces in piece
// order (the same result whichever CTA is last) with its own TMEM values,
// applies SiLU * up and stores the bf16 tile by TMA. It then clears the
// unit's ticket and flags for the next launch. No CTA waits for work that has
// not started: the last to draw waits only for pieces whose CTAs drew before.
// When that is the CTA's final segment, the other pieces' rows come in by
// bulk copies into the idle TMA ring; a non-last piece gives its TMEM back
// to the MMA warp before its stores drain. Slower than one unit per CTA at
// the Llama-3-8B shape (72.2 vs 62.1 us), so the host uses it only when asked
// (FOUNDRY_SWIGLU_SK=1).
namespace {

constexpr int SWIGLU_SK_MAXP = 3;  // pieces per unit (flags: ticket + one ready word per piece)

// Bulk (non-tensor) global -> shared copy, completion on `bar`; both
// addresses 16-byte aligned, bytes a multiple of 16. No multicast.
__device__ __forceinline__ void bulk_copy_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

template <int BN>
__device__ __forceinline__ void gemm_swiglu_sk_body(const CUtensorMap* tmA, const CUtensorMap* tmB,
                                                    const CUtensorMap* tmO, int M, int N, int K, int mode,
                                                    float* __restrict__ ws, int* __restrict__ flags) {
  using C = Cfg<BN, 2>;
  constexpr int STAGES = C::STAGES;
  constexpr int NBUF = C::ACC_BUFS;
  constexpr int EC = EPI_COLS;
  static_assert(BN % EC == 0, "epilogue chunks");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;                              // [STAGES][2][128 x 64]
  uint8_t* sB = smem + STAGES * 2 * C::A_BYTES;     // [STAGES][BN x 64]
  uint8_t* stg = smem + STAGES * C::STAGE_BYTES;    // epilogue tiles (STG_BYTES)
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * C::STAGE_BYTES + STG_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* ebar = tempty + 2;
  // Fix-up of the CTA's final segment: the other pieces' rows of one 32-column
  // chunk (gate 16 KB + up 16 KB) per slot of the then idle TMA ring.
  constexpr int PF_BYTES = 2 * EC * BM * 4;
  constexpr int PF_SLOTS = (STAGES * C::STAGE_BYTES) / PF_BYTES;
  static_assert(PF_SLOTS >= SWIGLU_SK_MAXP - 1, "one chunk of every other piece in flight");
  uint64_t* pbar = ebar + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(pbar + PF_SLOTS);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
  int* unit_ticket = abort_flag + 1;  // the ticket this CTA drew for its current unit

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int half = M / 2;  // up rows start here
  const int units = half / BM;
  const int KB = (K + BK - 1) / BK;
  const int G = gridDim.x;
  const long long T = static_cast<long long>(units) * KB;
  auto cta_start = [&](int b) -> long long { return T * b / G; };
  const long long it0 = cta_start(blockIdx.x);
  const long long it1 = cta_start(blockIdx.x + 1);
  // CTA whose range holds iteration i.
  auto cta_of = [&](long long i) -> int {
    int b = static_cast<int>(i * G / T);
    while (b + 1 < G && cta_start(b + 1) <= i) ++b;
    while (b > 0 && cta_start(b) > i) --b;
    return b;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 4);
    }
    mbar_init(ebar, 4);
    for (int q = 0; q < PF_SLOTS; ++q) mbar_init(&pbar[q], 1);
    *abort_flag = 0;
    fence_barrier_init();
    fence_proxy_async();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(tmA);
    tma_prefetch_desc(tmB);
    tma_prefetch_desc(tmO);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_trigger();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      const uint64_t pol = policy_evict_first();
      const int pf_dist = (mode >> 8) & 0xFF;
      auto load_a = [&](int st, int kb, int u) {
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
          uint8_t* dst = sA + (st * 2 + mt) * C::A_BYTES;
          const int row = mt * half + u * BM;
          if (mode & EPI_A_STREAM)
            tma_load_2d_hint(dst, tmA, &full[st], kb * BK, row, pol);
          else
            tma_load_2d(dst, tmA, &full[st], kb * BK, row);
        }
      };
      // The first segment's A tiles of the whole ring go out before the wait
      // for the previous kernel when A is the weights (EPI_A_CONST).
      int pre = 0;
      if ((mode & EPI_A_CONST) && it0 < it1) {
        const int u = static_cast<int>(it0 / KB);
        const int kb0 = static_cast<int>(it0 % KB);
        const int kb1 = static_cast<int>(min(static_cast<long long>(KB), kb0 + (it1 - it0)));
        pre = min(STAGES, kb1 - kb0);
        for (int i = 0; i < pre; ++i) {
          mbar_arrive_expect_tx(&full[i], C::STAGE_BYTES);
          load_a(i, kb0 + i, u);
        }
      }
      pdl_wait();
      bool first_seg = true;
      for (long long it = it0; it < it1 && !*(volatile int*)abort_flag;) {
        const int u = static_cast<int>(it / KB);
        const int kb0 = static_cast<int>(it % KB);
        const int kb1 = static_cast<int>(min(static_cast<long long>(KB), kb0 + (it1 - it)));
        for (int kb = kb0; kb < min(kb1, kb0 + pf_dist); ++kb)
#pragma unroll
          for (int mt = 0; mt < 2; ++mt) tma_prefetch_2d(tmA, kb * BK, mt * half + u * BM);
        bool stop = false;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (pf_dist && kb + pf_dist < kb1) {
#pragma unroll
            for (int mt = 0; mt < 2; ++mt) tma_prefetch_2d(tmA, (kb + pf_dist) * BK, mt * half + u * BM);
          }
          if (first_seg && kb - kb0 < pre) {
            // stage armed and its A tiles issued before pdl_wait
          } else {
            if (!mbar_wait(&empty[stage], phase ^ 1, FB_KERR_TIMEOUT_EMPTY)) {
              *(volatile int*)abort_flag = 1;
              stop = true;
              break;
            }
            mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
            load_a(stage, kb, u);
          }
          tma_load_2d(sB + stage * C::B_BYTES, tmB, &full[stage], kb * BK, 0);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (stop) break;
        first_seg = false;
        it += kb1 - kb0;
      }
      // Drain: every armed stage must complete before the CTA may exit.
      for (int s = 0; s < STAGES; ++s) {
        mbar_wait(&empty[stage], phase ^ 1, FB_KERR_TIMEOUT_EMPTY);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer: one accumulator pair per segment ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16<BM, BN>();
      int stage = 0;
      uint32_t phase = 0;
      int seg = 0;
      for (long long it = it0; it < it1 && !*(volatile int*)abort_flag; ++seg) {
        const int kb0 = static_cast<int>(it % KB);
        const int kb1 = static_cast<int>(min(static_cast<long long>(KB), kb0 + (it1 - it)));
        const int acc = NBUF == 2 ? (seg & 1) : 0;
        const uint32_t aphase = NBUF == 2 ? ((seg >> 1) & 1) : (seg & 1);
        if (!mbar_wait(&tempty[acc], aphase ^ 1, FB_KERR_TIMEOUT_TMEM)) {
          *(volatile int*)abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * C::ACC_COLS;
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, FB_KERR_TIMEOUT_FULL)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t bdesc = sdesc_sw128(smem_u32(sB + stage * C::B_BYTES));
#pragma unroll
          for (int mt = 0; mt < 2; ++mt) {
            const uint64_t adesc = sdesc_sw128(smem_u32(sA + (stage * 2 + mt) * C::A_BYTES));
#pragma unroll
            for (int k = 0; k < BK / 16; ++k)
              mma_bf16(d_tmem + mt * BN, adesc + (uint64_t)(k * 2), bdesc + (uint64_t)(k * 2), idesc,
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
        it += kb1 - kb0;
      }
    }
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    pdl_wait();  // flag and output writes follow the previous kernel
    const int quarter = warp & 3;
    const int et = threadIdx.x - 64;    // 0..127; 0 draws tickets and issues the tile stores
    const int f = quarter * 32 + lane;  // feature (TMEM lane) of this thread within the unit
    uint32_t ephase = 0, chunk = 0;
    bool ok = true;
    auto epi_sync = [&]() -> bool {
      __syncwarp();
      if (lane == 0) mbar_arrive(ebar);
      const bool done = mbar_wait(ebar, ephase, FB_KERR_TIMEOUT_TMEM);
      ephase ^= 1;
      return done;
    };
    // One piece's slot: gate then up, each [BN / 4][128 features][4 columns]
    // of fp32, so that a warp's float4 accesses of one column group are 512
    // contiguous bytes.
    constexpr size_t SLOT = static_cast<size_t>(2) * BM * BN;
    int seg = 0;
    for (long long it = it0; ok && it < it1 && !*(volatile int*)abort_flag; ++seg) {
      const int u = static_cast<int>(it / KB);
      const int kb0 = static_cast<int>(it % KB);
      const int kb1 = static_cast<int>(min(static_cast<long long>(KB), kb0 + (it1 - it)));
      it += kb1 - kb0;
      const int acc = NBUF == 2 ? (seg & 1) : 0;
      const uint32_t aphase = NBUF == 2 ? ((seg >> 1) & 1) : (seg & 1);
      if (!mbar_wait(&tfull[acc], aphase, FB_KERR_TIMEOUT_TMEM)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t t_g = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * C::ACC_COLS;
      const int first = cta_of(static_cast<long long>(u) * KB);
      const int npieces = cta_of(static_cast<long long>(u) * KB + KB - 1) - first + 1;
      const int piece = static_cast<int>(blockIdx.x) - first;
      if (npieces > SWIGLU_SK_MAXP) {  // the host sizes the grid so that this cannot happen
        set_status(FB_KERR_BAD_ARG);
        ok = false;
        break;
      }
      int* ticket = flags + u * (1 + SWIGLU_SK_MAXP);
      int* ready = ticket + 1;
      bool last = true;
      if (npieces > 1) {
        if (et == 0) *unit_ticket = atomicAdd(ticket, 1);
        if (!(ok = epi_sync())) break;
        last = *(volatile int*)unit_ticket == npieces - 1;
      }
      if (!last) {
        // fp32 gate and up rows of this piece: row f, BN contiguous floats each
        float4* slot = reinterpret_cast<float4*>(ws + static_cast<size_t>(u * SWIGLU_SK_MAXP + piece) * SLOT);
#pragma unroll 1
        for (int j = 0; j < 2; ++j) {
          float4* dst = slot + static_cast<size_t>(j) * (BM * BN / 4) + f;
#pragma unroll 1
          for (int c1 = 0; c1 < BN; c1 += EC) {
            uint32_t rr[EC];
#pragma unroll
            for (int q = 0; q < EC / 16; ++q)
              tmem_ld16(t_g + j * BN + c1 + 16 * q, *reinterpret_cast<uint32_t(*)[16]>(rr + 16 * q));
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < EC / 4; ++i)
              dst[(c1 / 4 + i) * BM] = make_float4(__uint_as_float(rr[4 * i]), __uint_as_float(rr[4 * i + 1]),
                                                   __uint_as_float(rr[4 * i + 2]), __uint_as_float(rr[4 * i + 3]));
          }
        }
        // The stores read registers: the accumulators go back to the MMA
        // warp now, and the next piece's MMAs overlap the stores' drain.
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[acc]);
        __threadfence();
        if (!(ok = epi_sync())) break;  // all 128 rows written
        if (et == 0) st_release_gpu(ready + piece, 1);
        continue;
      } else {
        // Last piece: the other pieces' rows must be in place (their CTAs drew
        // their tickets before this one; bounded wait for their flags).
        for (int q = 0; q < npieces && ok; ++q) {
          if (q == piece) continue;
          const uint64_t t0 = globaltimer();
          uint32_t spins = 0;
          while (ld_acquire_gpu(ready + q) == 0) {
            if ((++spins & 255u) == 0 && globaltimer() - t0 > FB_WAIT_NS) {
              set_status(FB_KERR_TIMEOUT_PEER);
              ok = false;
              break;
            }
          }
        }
        if (!ok) break;
        const float* slots = ws + static_cast<size_t>(u * SWIGLU_SK_MAXP) * SLOT;
        // After the CTA's final segment the ring is idle (its MMAs are done
        // and the producer issues nothing more): the other pieces' rows come
        // in by bulk copies, PF_SLOTS chunks ahead, instead of one dependent
        // L2 round trip per chunk and piece.
        const int nq = npieces - 1;
        const int items = (BN / EC) * nq;  // (chunk, other piece), chunk-major
        const bool staged = nq > 0 && it >= it1;
        int issued = 0, waited = 0;  // items issued (thread 0) / waited for (each thread)
        auto issue = [&](int i) {
          ++issued;
          const int c = i / nq, qi = i % nq;
          const int q = qi < piece ? qi : qi + 1;
          const int sl = i % PF_SLOTS;
          const float* src = slots + q * SLOT + static_cast<size_t>(c) * (EC * BM);
          uint8_t* dst = smem + sl * PF_BYTES;
          mbar_arrive_expect_tx(&pbar[sl], PF_BYTES);
          bulk_copy_g2s(dst, src, PF_BYTES / 2, &pbar[sl]);
          bulk_copy_g2s(dst + PF_BYTES / 2, src + BM * BN, PF_BYTES / 2, &pbar[sl]);
        };
        if (staged && et == 0) {
          asm volatile("fence.proxy.async.global;" ::: "memory");  // acquired rows -> bulk copy reads
          for (int i = 0; i < min(items, PF_SLOTS); ++i) issue(i);
        }
#pragma unroll 1
        for (int c1 = 0; c1 < BN && ok; c1 += EC, ++chunk) {
          const int buf = chunk & 1;
          bf16* sb = reinterpret_cast<bf16*>(stg) + buf * (EPI_COLS * BM);
          uint32_t rg[EC], ru[EC];
#pragma unroll
          for (int q = 0; q < EC / 16; ++q) {
            tmem_ld16(t_g + c1 + 16 * q, *reinterpret_cast<uint32_t(*)[16]>(rg + 16 * q));
            tmem_ld16(t_g + BN + c1 + 16 * q, *reinterpret_cast<uint32_t(*)[16]>(ru + 16 * q));
          }
          tmem_ld_wait();
          // sum of the pieces in piece order, this CTA's own from TMEM
          float g[EC], v[EC];
#pragma unroll
          for (int t = 0; t < EC; ++t) g[t] = v[t] = 0.f;
#pragma unroll 1
          for (int q = 0; q < npieces && ok; ++q) {
            if (q == piece) {
#pragma unroll
              for (int t = 0; t < EC; ++t) {
                g[t] += __uint_as_float(rg[t]);
                v[t] += __uint_as_float(ru[t]);
              }
            } else if (staged) {
              const int i = (c1 / EC) * nq + (q < piece ? q : q - 1);
              const int sl = i % PF_SLOTS;
              if (!(ok = mbar_wait(&pbar[sl], (i / PF_SLOTS) & 1, FB_KERR_TIMEOUT_FULL))) break;
              ++waited;
              const float4* pg = reinterpret_cast<const float4*>(smem + sl * PF_BYTES) + f;
              const float4* pu = pg + PF_BYTES / 2 / 16;
#pragma unroll
              for (int i4 = 0; i4 < EC / 4; ++i4) {
                const float4 a = pg[i4 * BM], b = pu[i4 * BM];
                g[4 * i4] += a.x;
                g[4 * i4 + 1] += a.y;
                g[4 * i4 + 2] += a.z;
                g[4 * i4 + 3] += a.w;
                v[4 * i4] += b.x;
                v[4 * i4 + 1] += b.y;
                v[4 * i4 + 2] += b.z;
                v[4 * i4 + 3] += b.w;
              }
            } else {
              const float4* pg = reinterpret_cast<const float4*>(slots + q * SLOT) + (c1 / 4) * BM + f;
              const float4* pu = pg + BM * BN / 4;
#pragma unroll
              for (int i = 0; i < EC / 4; ++i) {
                const float4 a = __ldcg(pg + i * BM), b = __ldcg(pu + i * BM);
                g[4 * i] += a.x;
                g[4 * i + 1] += a.y;
                g[4 * i + 2] += a.z;
                g[4 * i + 3] += a.w;
                v[4 * i] += b.x;
                v[4 * i + 1] += b.y;
                v[4 * i + 2] += b.z;
                v[4 * i + 3] += b.w;
              }
            }
          }
          if (!ok) break;
          if (et == 0 && chunk >= 2) bulk_wait_read_1();  // this buffer's previous store has read it
          if (!(ok = epi_sync())) break;
          if (staged && et == 0) {  // every thread has read this chunk's slots: refill them
            for (int qi = 0; qi < nq; ++qi) {
              const int i = (c1 / EC) * nq + qi + PF_SLOTS;
              if (i < items) issue(i);
            }
          }
#pragma unroll
          for (int t = 0; t < EC; ++t) sb[t * BM + f] = f2bf(g[t] / (1.f + __expf(-g[t])) * v[t]);
          fence_proxy_async();  // generic-proxy writes -> visible to the TMA engine
          if (!(ok = epi_sync())) break;
          if (et == 0) {
            tma_store_2d(tmO, sb, u * BM, c1);
            bulk_commit();
          }
        }
        // Copies still in flight after an error land before the CTA exits
        // (bounded waits; items are issued and waited for in order).
        if (staged && et == 0)
          for (int i = waited; i < issued; ++i) mbar_wait(&pbar[i % PF_SLOTS], (i / PF_SLOTS) & 1, FB_KERR_TIMEOUT_FULL);
        // every piece has been read: clear the unit's counters for the next launch
        if (ok && npieces > 1 && et == 0) {
          *ticket = 0;
          for (int q = 0; q < npieces; ++q) ready[q] = 0;
        }
      }
      if (!ok) break;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
    if (!ok) *(volatile int*)abort_flag = 1;
    if (et == 0) bulk_wait_all();  // the tile stores have read shared memory and landed
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, C::TMEM_COLS);
}

}  // namespace

#define FB_GEMM_SWIGLU_SK_INSTANCE(BN)                                                                              \
  extern "C" __global__ void __launch_bounds__(NUM_THREADS, 1) fb_gemm_swiglu_sk_bn##BN(                            \
      const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,                             \
      const __grid_constant__ CUtensorMap tmO, int M, int N, int K, int mode, float* ws, int* flags) {              \
    gemm_swiglu_sk_body<BN>(&tmA, &tmB, &tmO, M, N, K, mode, ws, flags);                                            \
  }

FB_GEMM_SWIGLU_SK_INSTANCE(256)

// ==== two-SM variant (cta_group::2) ======================================================
//
// fb_gemm2_bf16_bn{BN}: a cluster of two CTAs (the two SMs of a TPC) computes
// one 256-row x BN tile. Each CTA loads its own 128 A rows and half of the BN
// B rows into its shared memory; the even CTA issues tcgen05.mma.cta_group::2
// (M = 256), which reads both CTAs' shared memory at the same offsets and
// accumulates each CTA's 128 rows x BN in that CTA's TMEM. Per SM and k-block
// that is 16 KB of A + BN/2 x 128 B of B instead of 16 KB + BN x 128 B for the
// same tensor work, so the ring is deeper at the same shared memory.
//
// Cross-CTA synchronisation (addresses of the other CTA come from mapa):
//   full[s]   even CTA only: one arrival (its producer, expecting both CTAs'
//             bytes); both CTAs' TMA loads complete_tx on it
//   empty[s]  each CTA: the even CTA's MMA commits arrive on both
//   tfull[a]  each CTA: the even CTA commits on both after a unit's last k-block
//   tempty[a] even CTA only: 8 arrivals, the 4 epilogue warps of each CTA
// Every mbarrier wait is bounded; the cluster barriers at start (barrier
// initialisation visible to the peer) and end (no CTA leaves while the pair's
// MMAs or remote arrivals may still touch it) are reached on every path.
// No TMA multicast: loads carry .cta_group::2 only.
namespace {

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t mapa_cta(const void* p, uint32_t rank) {
  uint32_t d;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(d) : "r"(smem_u32(p)), "r"(rank));
  return d;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const void* tmap, uint32_t bar, int32_t c0, int32_t c1,
                                                 uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(c0), "r"(c1), "r"(bar), "l"(policy)
      : "memory");
}
__device__ __forceinline__ void mma_bf16_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(
          tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}
__device__ __forceinline__ void mma_commit_pair(uint32_t bar_cluster) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar_cluster)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols));
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}

template <int BN>
struct PairCfg {
  static constexpr int A_BYTES = BM * BK * 2;        // this CTA's 128 A rows per K step
  static constexpr int B_BYTES = (BN / 2) * BK * 2;  // this CTA's half of the B rows
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (192 * 1024) / STAGE_BYTES > 8 ? 8 : (192 * 1024) / STAGE_BYTES;
  static constexpr int ACC_BUFS = (2 * BN <= 512) ? 2 : 1;
  static constexpr uint32_t TMEM_COLS = tmem_cols_for(ACC_BUFS * BN);
};

template <int BN>
__device__ __forceinline__ void gemm_pair_body(const CUtensorMap* tmA, const CUtensorMap* tmB, const CUtensorMap* tmO,
                                               const CUtensorMap* tmR, bf16* __restrict__ out,
                                               const bf16* residual, int M, int N, int K, int ldo, int mode,
                                               int splits, float* __restrict__ ws, long long split_stride) {
  using C = PairCfg<BN>;
  constexpr int STAGES = C::STAGES;
  constexpr int NBUF = C::ACC_BUFS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;                           // [STAGES][128 x 64]
  uint8_t* sB = smem + STAGES * C::A_BYTES;     // [STAGES][BN/2 x 64]
  uint8_t* stg = smem + STAGES * C::STAGE_BYTES;  // epilogue tiles of this CTA (STG_BYTES)
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * C::STAGE_BYTES + STG_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* ebar = tempty + 2;  // this CTA's four epilogue warps' rendezvous
  uint64_t* rbar = ebar + 1;    // residual tile loads, one per buffer
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(rbar + 2);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();  // 0: issues the MMAs; 1: its peer
  const int pair = blockIdx.x >> 1, num_pairs = gridDim.x >> 1;
  const int num_m = (M + 2 * BM - 1) / (2 * BM);
  const int num_n = (N + BN - 1) / BN;
  const int KB = (K + BK - 1) / BK;
  const int kb_per = (KB + splits - 1) / splits;
  const int num_units = num_m * num_n * splits;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 8);
    }
    mbar_init(ebar, 4);
    mbar_init(&rbar[0], 1);
    mbar_init(&rbar[1], 1);
    *abort_flag = 0;
    fence_barrier_init();
    fence_proxy_async();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(tmA);
    tma_prefetch_desc(tmB);
    if (mode & EPI_TMA_OUT) {
      tma_prefetch_desc(tmO);
      if (mode & EPI_RESIDUAL) tma_prefetch_desc(tmR);
    }
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, C::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // both CTAs' barriers initialised before either signals the other
  tc_fence_after();
  pdl_trigger();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs) ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      const uint64_t pol_a = (mode & EPI_A_STREAM) ? policy_evict_first() : policy_evict_last();
      const uint64_t pol_b = (mode & EPI_B_STREAM) ? policy_evict_first() : policy_evict_last();
      const int pf_dist = (mode >> 8) & 0xFF;
      // Before waiting for the previous kernel: the first unit's weight (A)
      // tiles of the whole ring, when no kernel of the step writes A
      // (EPI_A_CONST); the token tiles (B) follow pdl_wait.
      int pre = 0;
      if ((mode & EPI_A_CONST) && pair < num_units) {
        const int mn = pair / splits, sp = pair % splits;
        const int kb0 = sp * kb_per, kb1 = min(KB, kb0 + kb_per);
        const int a_row = (mn % num_m) * 2 * BM + rank * BM;
        pre = min(STAGES, kb1 - kb0);
        for (int i = 0; i < pre; ++i) {
          if (rank == 0) mbar_arrive_expect_tx(&full[i], 2 * C::STAGE_BYTES);
          tma_load_2d_pair(sA + i * C::A_BYTES, tmA, mapa_cta(&full[i], 0), (kb0 + i) * BK, a_row, pol_a);
        }
      }
      pdl_wait();
      for (int u = pair; u < num_units && !*(volatile int*)abort_flag; u += num_pairs) {
        const int mn = u / splits, sp = u % splits;
        const int m_blk = mn % num_m, n_blk = mn / num_m;
        const int kb0 = sp * kb_per, kb1 = min(KB, kb0 + kb_per);
        const int a_row = m_blk * 2 * BM + rank * BM;
        const int b_row = n_blk * BN + rank * (BN / 2);
        for (int kb = kb0; kb < min(kb1, kb0 + pf_dist); ++kb) tma_prefetch_2d(tmA, kb * BK, a_row);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (pf_dist && kb + pf_dist < kb1) tma_prefetch_2d(tmA, (kb + pf_dist) * BK, a_row);
          const uint32_t bar = mapa_cta(&full[stage], 0);
          if (!(u == pair && kb - kb0 < pre)) {  // else armed, A issued before pdl_wait
            if (!mbar_wait(&empty[stage], phase ^ 1, FB_KERR_TIMEOUT_EMPTY)) {
              *(volatile int*)abort_flag = 1;
              break;
            }
            if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * C::STAGE_BYTES);
            tma_load_2d_pair(sA + stage * C::A_BYTES, tmA, bar, kb * BK, a_row, pol_a);
          }
          tma_load_2d_pair(sB + stage * C::B_BYTES, tmB, bar, kb * BK, b_row, pol_b);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // Drain: every stage this CTA armed is consumed before it may leave.
      for (int s = 0; s < STAGES; ++s) {
        mbar_wait(&empty[stage], phase ^ 1, FB_KERR_TIMEOUT_EMPTY);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (even CTA) ----------------
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = idesc_bf16<2 * BM, BN>();
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      for (int u = pair; u < num_units && !*(volatile int*)abort_flag; u += num_pairs, ++it) {
        const int sp = u % splits;
        const int kb0 = sp * kb_per, kb1 = min(KB, kb0 + kb_per);
        const int acc = NBUF == 2 ? (it & 1) : 0;
        const uint32_t aphase = NBUF == 2 ? ((it >> 1) & 1) : (it & 1);
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
          for (int k = 0; k < BK / 16; ++k)
            mma_bf16_pair(d_tmem, adesc + (uint64_t)(k * 2), bdesc + (uint64_t)(k * 2), idesc,
                          (kb > kb0 || k > 0) ? 1u : 0u);
          mma_commit_pair(mapa_cta(&empty[stage], 0));
          mma_commit_pair(mapa_cta(&empty[stage], 1));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        mma_commit_pair(mapa_cta(&tfull[acc], 0));
        mma_commit_pair(mapa_cta(&tfull[acc], 1));
        if (!ok) {
          *(volatile int*)abort_flag = 1;
          break;
        }
      }
    }
  } else {
    // ---------------- epilogue (warps 2..5 of both CTAs) ----------------
    pdl_wait();  // residual reads and output writes follow the previous kernel
    const int quarter = warp & 3;
    const uint32_t tempty0 = mapa_cta(&tempty[0], 0), tempty1 = mapa_cta(&tempty[1], 0);
    const int et = threadIdx.x - 64;  // 0..127; 0 issues this CTA's tile stores
    const bool tma_out = (mode & EPI_TMA_OUT) && (mode & EPI_TRANSPOSE);
    uint32_t ephase = 0, rphase = 0, chunk = 0;
    bool ok = true;
    auto epi_sync = [&]() -> bool {
      __syncwarp();
      if (lane == 0) mbar_arrive(ebar);
      const bool done = mbar_wait(ebar, ephase, FB_KERR_TIMEOUT_TMEM);
      ephase ^= 1;
      return done;
    };
    int it = 0;
    for (int u = pair; u < num_units && !*(volatile int*)abort_flag; u += num_pairs, ++it) {
      const int mn = u / splits, sp = u % splits;
      const int m_blk = mn % num_m, n_blk = mn / num_m;
      const int acc = NBUF == 2 ? (it & 1) : 0;
      const uint32_t aphase = NBUF == 2 ? ((it >> 1) & 1) : (it & 1);
      if (!mbar_wait(&tfull[acc], aphase, FB_KERR_TIMEOUT_TMEM)) {
        *(volatile int*)abort_flag = 1;
        break;
      }
      tc_fence_after();
      float* part = splits > 1 ? ws + static_cast<size_t>(sp) * split_stride : nullptr;
      const int gm = m_blk * 2 * BM + rank * BM + quarter * 32 + lane;  // D row of this thread
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * BN;
      if (tma_out) {
        // Staged TMA-store epilogue (as fb_gemm_bf16): per 32-token chunk a
        // [32 tokens][128 features] tile of this CTA's rows, double-buffered.
        constexpr int EC = BN < EPI_COLS ? BN : EPI_COLS;
        const int gm0 = m_blk * 2 * BM + rank * BM;
        const int f = quarter * 32 + lane;
#pragma unroll 1
        for (int c1 = 0; c1 < BN && ok; c1 += EC, ++chunk) {
          const int buf = chunk & 1;
          const int gn0 = n_blk * BN + c1;
          float* sf = reinterpret_cast<float*>(stg) + buf * (EPI_COLS * BM);
          bf16* sb = reinterpret_cast<bf16*>(stg) + buf * (EPI_COLS * BM);
          bf16* sr = reinterpret_cast<bf16*>(stg + STG_BYTES / 2) + buf * (EPI_COLS * BM);
          uint32_t rr[EC];
#pragma unroll
          for (int j = 0; j < EC / 16; ++j)
            tmem_ld16(t_row + c1 + 16 * j, *reinterpret_cast<uint32_t(*)[16]>(rr + 16 * j));
          tmem_ld_wait();
          if (et == 0 && chunk >= 2) bulk_wait_read_1();  // this buffer's previous store has read it
          if (!(ok = epi_sync())) break;
          if (!part && (mode & EPI_RESIDUAL)) {
            if (et == 0) {
              mbar_arrive_expect_tx(&rbar[buf], EC * BM * 2);
              tma_load_2d(sr, tmR, &rbar[buf], gm0, gn0);
            }
            if (!(ok = mbar_wait(&rbar[buf], (rphase >> buf) & 1u, FB_KERR_TIMEOUT_FULL))) break;
            rphase ^= 1u << buf;
          }
          if (part) {
#pragma unroll
            for (int t = 0; t < EC; ++t) sf[t * BM + f] = __uint_as_float(rr[t]);
          } else if (mode & EPI_RESIDUAL) {
#pragma unroll
            for (int t = 0; t < EC; ++t) sb[t * BM + f] = f2bf(__uint_as_float(rr[t]) + bf2f(sr[t * BM + f]));
          } else {
#pragma unroll
            for (int t = 0; t < EC; ++t) sb[t * BM + f] = f2bf(__uint_as_float(rr[t]));
          }
          fence_proxy_async();  // generic-proxy writes -> visible to the TMA engine
          if (!(ok = epi_sync())) break;
          if (et == 0) {
            if (part)
              tma_store_3d(tmO, sf, gm0, gn0, sp);
            else
              tma_store_2d(tmO, sb, gm0, gn0);
            bulk_commit();
          }
        }
        if (!ok) {
          *(volatile int*)abort_flag = 1;
          break;
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(acc ? tempty1 : tempty0);
        continue;
      }
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 16) {
        uint32_t r[16];
        tmem_ld16(t_row + c0, r);
        tmem_ld_wait();
        const int gn0 = n_blk * BN + c0;
        if (gm >= M) continue;
        if (mode & EPI_TRANSPOSE) {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int gn = gn0 + i;
            if (gn < N) {
              const size_t idx = static_cast<size_t>(gn) * ldo + gm;
              float v = __uint_as_float(r[i]);
              if (part) {
                part[idx] = v;
              } else {
                if (mode & EPI_RESIDUAL) v += bf2f(residual[idx]);
                out[idx] = f2bf(v);
              }
            }
          }
        } else {
          const size_t base = static_cast<size_t>(gm) * ldo + gn0;
#pragma unroll
          for (int i = 0; i < 16; ++i)
            if (gn0 + i < N) {
              float v = __uint_as_float(r[i]);
              if (part) {
                part[base + i] = v;
              } else {
                if (mode & EPI_RESIDUAL) v += bf2f(residual[base + i]);
                out[base + i] = f2bf(v);
              }
            }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc ? tempty1 : tempty0);
    }
    if (et == 0 && tma_out) bulk_wait_all();  // the tile stores have read shared memory and landed
  }

  tc_fence_before();
  cluster_sync_all();  // the pair's MMAs, commits and remote arrivals are done
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
}

}  // namespace

#define FB_GEMM_PAIR_INSTANCE(BN)                                                                                   \
  extern "C" __global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NUM_THREADS, 1) fb_gemm2_bf16_bn##BN(      \
      const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,                             \
      const __grid_constant__ CUtensorMap tmO, const __grid_constant__ CUtensorMap tmR, bf16* out,                  \
      const bf16* residual, int M, int N, int K, int ldo, int mode, int splits, float* ws,                          \
      long long split_stride) {                                                                                      \
    gemm_pair_body<BN>(&tmA, &tmB, &tmO, &tmR, out, residual, M, N, K, ldo, mode, splits, ws, split_stride);       \
  }

FB_GEMM_PAIR_INSTANCE(64)
FB_GEMM_PAIR_INSTANCE(128)
FB_GEMM_PAIR_INSTANCE(256)
