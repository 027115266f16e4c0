// Causal prefill attention on the tcgen05 tensor cores (head_dim 128, bf16,
// GQA, packed variable-length prompts).
//
// CTA = (128-query tile of one prompt, query head). Per 128-key tile j of the
// prompt (tiles past the causal diagonal are skipped):
//   S_j = Q K_j^T      tcgen05.mma M=128 (queries) N=128 (keys) K=128 into one
//                      of two TMEM S buffers (QK of tile j+1 overlaps the
//                      softmax of tile j)
//   softmax            4 warps, thread r owns query row r: running max m and
//                      sum l in registers, p = exp2(s - m) written as bf16 to
//                      a 128B-swizzled K-major P tile in shared memory
//   O += P_j V_j       tcgen05.mma M=128 N=128 (head dims) K=128 (keys), V read
//                      MN-major from the TMA image; O stays in TMEM and a
//                      warp rescales its 32 rows (tcgen05.ld/st) only when one
//                      of its row maxima moved
// Epilogue: O / l -> bf16, one 256-byte row per thread.
//
// Roles: warp 0 TMA producer (Q once, K/V through a 2-stage ring), warp 1
// TMEM owner + MMA issuer, warps 2..5 softmax + epilogue. Tensor maps cover
// exactly the chunk's rows, so rows past the end read as zeros. No TMA
// multicast; every wait bounded (fb_common.cuh).
#include "fb_common.cuh"

FB_DEFINE_STATUS

using namespace fbk;

namespace {

constexpr int D = 128;
constexpr int BQ = 128;   // queries per tile
constexpr int BKV = 128;  // keys per tile
constexpr int HALF = BQ * 128;          // one 64-dim half of a 128-row tile: 128 rows x 128 B
constexpr int TILE = 2 * HALF;           // 128 rows x 128 dims bf16
constexpr int STAGES = 2;
constexpr float RESCALE_LOG2 = 8.f;  // lazy-rescale threshold (log2 units: p <= 256)

struct Smem {
  uint8_t q[TILE];
  uint8_t kv[STAGES][2 * TILE];  // K then V
  uint8_t p[TILE];
  uint64_t q_full, kv_full[STAGES], kv_empty[STAGES];
  uint64_t s_full[2], s_empty[2], p_full, o_full;
  uint32_t tmem;
  int abort;
};
static_assert(sizeof(Smem) + 1024 <= 200 * 1024, "host requests 200 KB of dynamic shared memory");

__device__ __forceinline__ uint64_t desc_mn(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFF) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFF) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }


// Byte offset of (row, col) in a K-major [128 rows x 128 cols] bf16 tile stored
// as two 64-column halves with the 128-byte swizzle.
__device__ __forceinline__ uint32_t sw_offset(int row, int col) {
  return (col >> 6) * HALF + row * 128 + ((((col & 63) >> 3) ^ (row & 7)) << 4) + (col & 7) * 2;
}

}  // namespace

// q [T, Hq * 128] (tmQ), k, v [T, Hkv * 128] (tmK, tmV): tensor maps over the
// chunk's T rows, boxes of 64 dims x 128 rows, 128B swizzle. Work item =
// blockIdx.x -> (query tile tile_seq/tile_start of 128 rows, head
// blockIdx.y). out [T, ld_o] bf16 (head h at columns h * 128).
extern "C" __global__ void __launch_bounds__(192, 1) fb_prefill_attn_tc(
    const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
    const __grid_constant__ CUtensorMap tmV, bf16* __restrict__ out, int ld_o, const int* __restrict__ cu_seqlens,
    const int* __restrict__ tile_seq, const int* __restrict__ tile_start, int Hq, int Hkv, float scale_log2) {
  pdl_entry();
  extern __shared__ uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int head = blockIdx.y, kvh = head / (Hq / Hkv);
  const int seq = tile_seq[blockIdx.x];
  const int s0 = cu_seqlens[seq], s1 = cu_seqlens[seq + 1];
  const int qp0 = tile_start[blockIdx.x];  // first query position inside the prompt
  const int q0 = s0 + qp0;                 // first query row (packed)
  const int n_kt = (min(qp0 + BQ, s1 - s0) + BKV - 1) / BKV;  // key tiles up to the diagonal

  if (threadIdx.x == 0) {
    mbar_init(&sm.q_full, 1);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&sm.kv_full[s], 1);
      mbar_init(&sm.kv_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sm.s_full[b], 1);
      mbar_init(&sm.s_empty[b], 4);
    }
    mbar_init(&sm.p_full, 4);
    mbar_init(&sm.o_full, 1);
    sm.abort = 0;
    fence_barrier_init();
    fence_proxy_async();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(&sm.tmem, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem;
  const uint32_t t_o = tmem + 256;  // S buffers at columns 0 and 128

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      mbar_arrive_expect_tx(&sm.q_full, TILE);
      tma_load_2d(sm.q, &tmQ, &sm.q_full, head * D, q0);
      tma_load_2d(sm.q + HALF, &tmQ, &sm.q_full, head * D + 64, q0);
      for (int j = 0; j < n_kt; ++j) {
        const int st = j % STAGES;
        if (!mbar_wait(&sm.kv_empty[st], ((j / STAGES) & 1) ^ 1, FB_KERR_TIMEOUT_EMPTY)) {
          sm.abort = 1;
          break;
        }
        mbar_arrive_expect_tx(&sm.kv_full[st], 2 * TILE);
        const int row = s0 + j * BKV;
        uint8_t* kb = sm.kv[st];
        tma_load_2d(kb, &tmK, &sm.kv_full[st], kvh * D, row);
        tma_load_2d(kb + HALF, &tmK, &sm.kv_full[st], kvh * D + 64, row);
        tma_load_2d(kb + TILE, &tmV, &sm.kv_full[st], kvh * D, row);
        tma_load_2d(kb + TILE + HALF, &tmV, &sm.kv_full[st], kvh * D + 64, row);
      }
      for (int j = n_kt; j < n_kt + STAGES; ++j)  // drain
        mbar_wait(&sm.kv_empty[j % STAGES], ((j / STAGES) & 1) ^ 1, FB_KERR_TIMEOUT_EMPTY);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t id_qk = idesc_bf16<128, 128>();
      constexpr uint32_t id_pv = idesc_bf16<128, 128>() | (1u << 16);  // B (V) MN-major
      const uint32_t qb = smem_u32(sm.q), pb = smem_u32(sm.p);
      bool ok = mbar_wait(&sm.q_full, 0, FB_KERR_TIMEOUT_FULL);
      auto issue_qk = [&](int j) -> bool {
        const int st = j % STAGES, sb = j & 1;
        if (!mbar_wait(&sm.kv_full[st], (j / STAGES) & 1, FB_KERR_TIMEOUT_FULL) ||
            !mbar_wait(&sm.s_empty[sb], ((j >> 1) & 1) ^ 1, FB_KERR_TIMEOUT_TMEM))
          return false;
        tc_fence_after();
        const uint32_t kb = smem_u32(sm.kv[st]);
#pragma unroll
        for (int k = 0; k < 8; ++k) {  // K = 128 head dims, 16 per MMA
          const uint32_t h = k >> 2, off = (k & 3) * 32;
          mma_bf16(tmem + sb * 128, sdesc_sw128(qb + h * HALF + off), sdesc_sw128(kb + h * HALF + off), id_qk,
                   k > 0 ? 1u : 0u);
        }
        mma_commit(&sm.s_full[sb]);
        return true;
      };
      if (ok && n_kt > 0) ok = issue_qk(0);
      for (int j = 0; ok && j < n_kt; ++j) {
        if (j + 1 < n_kt && !issue_qk(j + 1)) {
          ok = false;
          break;
        }
        if (!mbar_wait(&sm.p_full, j & 1, FB_KERR_TIMEOUT_TMEM)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t vb = smem_u32(sm.kv[j % STAGES]) + TILE;
#pragma unroll
        for (int k = 0; k < 8; ++k) {  // K = 128 keys, 16 per MMA
          const uint32_t h = k >> 2, off = (k & 3) * 32;
          mma_bf16(t_o, sdesc_sw128(pb + h * HALF + off), desc_mn(vb + k * 2048, HALF, 1024), id_pv,
                   (j > 0 || k > 0) ? 1u : 0u);
        }
        mma_commit(&sm.o_full);
        mma_commit(&sm.kv_empty[j % STAGES]);
      }
      if (!ok) sm.abort = 1;
    }
  } else {
    // ---------------- softmax + epilogue (warps 2..5) ----------------
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // query row of this thread
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const int qpos = qp0 + r;             // position inside the prompt
    const bool qvalid = q0 + r < s1;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kt; ++j) {
      const int sb = j & 1;
      if (!mbar_wait(&sm.s_full[sb], (j >> 1) & 1, FB_KERR_TIMEOUT_TMEM)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t t_s = tmem + sb * 128 + lane_base;
      const int kpos0 = j * BKV;  // key positions of this tile: kpos0 + c
      // pass 1: row max over the valid keys (64 columns per TMEM round trip)
      float mx = -INFINITY;
#pragma unroll 1
      for (int c1 = 0; c1 < BKV; c1 += 64) {
        uint32_t sr[64];
#pragma unroll
        for (int q = 0; q < 4; ++q) tmem_ld16(t_s + c1 + 16 * q, *reinterpret_cast<uint32_t(*)[16]>(sr + 16 * q));
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          const int kp = kpos0 + c1 + i;
          if (qvalid && kp <= qpos) mx = fmaxf(mx, __uint_as_float(sr[i]) * scale_log2);
        }
      }
      // Lazy rescaling: the running max of a row moves (and O is rescaled)
      // only when the tile's max exceeds it by more than RESCALE_LOG2; until
      // then p = exp2(s - m) stays below 2^RESCALE_LOG2, exact in the fp32
      // sums. A warp rescales its O rows only if one of them moved.
      const float m_new = (mx > m_run + RESCALE_LOG2 || m_run == -INFINITY) ? fmaxf(m_run, mx) : m_run;
      const float m_use = m_new == -INFINITY ? 0.f : m_new;
      const float alpha = exp2f(m_run - m_use);  // 0 on the first tile (m_run = -inf), else 1 unless moved
      // P_j may only be written once PV_{j-1} has consumed P_{j-1}; O is
      // rescaled in place before PV_j accumulates into it.
      if (j > 0) {
        if (!mbar_wait(&sm.o_full, (j - 1) & 1, FB_KERR_TIMEOUT_TMEM)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll 1
          for (int c1 = 0; c1 < D; c1 += 64) {
            uint32_t orr[64];
#pragma unroll
            for (int q = 0; q < 4; ++q)
              tmem_ld16(t_o + lane_base + c1 + 16 * q, *reinterpret_cast<uint32_t(*)[16]>(orr + 16 * q));
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 64; ++i) orr[i] = __float_as_uint(__uint_as_float(orr[i]) * alpha);
#pragma unroll
            for (int q = 0; q < 4; ++q)
              tmem_st16(t_o + lane_base + c1 + 16 * q, *reinterpret_cast<const uint32_t(*)[16]>(orr + 16 * q));
          }
          tmem_st_wait();
        }
      }
      // pass 2: p = exp2(s - m), row sum, P row to shared memory
      float rs = 0.f;
#pragma unroll 1
      for (int c1 = 0; c1 < BKV; c1 += 64) {
        uint32_t sr[64];
#pragma unroll
        for (int q = 0; q < 4; ++q) tmem_ld16(t_s + c1 + 16 * q, *reinterpret_cast<uint32_t(*)[16]>(sr + 16 * q));
        tmem_ld_wait();
#pragma unroll
        for (int c2 = 0; c2 < 64; c2 += 16) {
          const int c0 = c1 + c2;
          float p[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int kp = kpos0 + c0 + i;
            p[i] = (qvalid && kp <= qpos) ? exp2f(__uint_as_float(sr[c2 + i]) * scale_log2 - m_use) : 0.f;
            rs += p[i];
          }
          uint4 lo, hi;
          bf162* l2 = reinterpret_cast<bf162*>(&lo);
          bf162* h2 = reinterpret_cast<bf162*>(&hi);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            l2[i] = __floats2bfloat162_rn(p[2 * i], p[2 * i + 1]);
            h2[i] = __floats2bfloat162_rn(p[8 + 2 * i], p[8 + 2 * i + 1]);
          }
          *reinterpret_cast<uint4*>(sm.p + sw_offset(r, c0)) = lo;
          *reinterpret_cast<uint4*>(sm.p + sw_offset(r, c0 + 8)) = hi;
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.s_empty[sb]);  // S buffer free for QK_{j+2}
      l_run = l_run * alpha + rs;
      m_run = m_new;
      fence_proxy_async();  // P (generic-proxy stores) -> visible to the tensor core
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.p_full);
    }
    if (ok && n_kt > 0 && mbar_wait(&sm.o_full, (n_kt - 1) & 1, FB_KERR_TIMEOUT_TMEM)) {
      tc_fence_after();
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      bf16* orow = out + static_cast<size_t>(q0 + r) * ld_o + head * D;
#pragma unroll 1
      for (int c0 = 0; c0 < D; c0 += 16) {
        uint32_t orr[16];
        tmem_ld16(t_o + lane_base + c0, orr);
        tmem_ld_wait();
        if (qvalid) {
          float f[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) f[i] = __uint_as_float(orr[i]) * inv;
          float a[8], b[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            a[i] = f[i];
            b[i] = f[8 + i];
          }
          *reinterpret_cast<uint4*>(orow + c0) = pack8(a);
          *reinterpret_cast<uint4*>(orow + c0 + 8) = pack8(b);
        }
      }
    } else if (!ok) {
      sm.abort = 1;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}
