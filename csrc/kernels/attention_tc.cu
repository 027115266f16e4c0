// Paged GQA decode attention on the tcgen05 tensor cores (head_dim 128,
// bf16 K/V pages of 64 tokens, fp32 softmax state).
//
// Work item = (sequence b, KV head, split). For each 128-token chunk (two
// pages) of the item:
//   S^T[tok, h]  = K[tok, :] . Q[h, :]      tcgen05.mma M=128 (tokens) N=16 (heads, G
//                                           real + zero padding) K=128, K-major A and B
//   softmax      4 warps, one TMEM lane (token) per thread: masked scores,
//                per-head running max over the chunk, p = exp2(s - m), P^T
//                written to shared memory in the 128B-swizzled K-major layout
//   O^T[d, h]    = V^T[d, tok] . P^T[tok, h] tcgen05.mma M=128 (dims) N=16 K=128
//                with V^T read MN-major from the same shared-memory image the
//                K-major TMA load produced
//   O            accumulated in registers (one TMEM lane = one head dim per
//                thread): o = o * alpha + O^T_chunk
// K/V pages stream through TMA (64 KB per chunk): one stage per CTA with
// three CTAs per SM (default), or a 3-stage ring with one CTA per SM; K and V
// have their own full/empty barriers, so the next chunk's K loads while this
// chunk's softmax and PV run. Only the live tokens of a sequence's last page
// are loaded (16-token row boxes). The grid is persistent and walks work
// items, so the producer runs ahead across item boundaries. Each live KV byte
// is read from HBM once per decode step.
//
// Roles: warp 0 TMA producer, warp 1 TMEM owner + MMA issuer, warps 2..5
// softmax/epilogue. No TMA multicast. All waits bounded (fb_common.cuh).
#include "fb_common.cuh"

FB_DEFINE_STATUS

using namespace fbk;

namespace {

constexpr int D = 128;
constexpr int PAGE = 64;
constexpr int CHUNK = 128;       // tokens per MMA chunk (two pages)
constexpr int NH = 16;           // padded head count (MMA N)
constexpr int BOX_BYTES = 64 * 128;              // 64 tokens x 64 dims x 2 B
constexpr int SUB_BYTES = 16 * 128;              // 16 tokens x 64 dims x 2 B (tail boxes)
constexpr int KV_BYTES = 2 * 2 * BOX_BYTES;      // one chunk of K (or V): 2 pages x 2 dim-halves
constexpr int STAGE_BYTES = 2 * KV_BYTES;        // K + V
constexpr int HALF_STRIDE = 2 * BOX_BYTES;       // dim-half block: 128 tokens x 128 B
constexpr int QP_BYTES = 2 * NH * 128;           // [2 halves][16 rows][128 B]

template <int STAGES>
struct Smem {
  uint8_t kv[STAGES][STAGE_BYTES];  // per stage: K [half][128 tok][128B], V same
  uint8_t q[QP_BYTES];
  uint8_t p[QP_BYTES];
  // K and V of a stage fill and drain separately: the next chunk's K loads
  // while this chunk's softmax and PV run.
  uint64_t kfull[STAGES], vfull[STAGES], kempty[STAGES], vempty[STAGES];
  uint64_t s_full, s_empty, p_full, o_full, o_empty, q_ready;
  float red_max[4][8];
  float red_l[4][8];
  float alpha[8];  // this chunk's rescale factor per head (the same in every softmax thread)
  float mrun[2][8];  // running max per head, by chunk parity (uniform across the softmax threads)
  uint32_t tmem;
  int abort;
};
static_assert(sizeof(Smem<3>) + 1024 <= 212992, "host requests 208 KB of dynamic shared memory (3 stages)");
static_assert(sizeof(Smem<1>) + 1024 <= 75776, "host requests 74 KB of dynamic shared memory (1 stage, 3 CTAs/SM)");

// K-major, 128B-swizzled descriptor with a given stride-byte-offset.
__device__ __forceinline__ uint64_t desc_kmajor(uint32_t saddr) { return sdesc_sw128(saddr); }

// MN-major, 128B-swizzled: LBO = stride between 64-element MN blocks, SBO =
// stride between 8-row K groups.
__device__ __forceinline__ uint64_t desc_mnmajor(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFF) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFF) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

// M=128, N=16, bf16 in, f32 accumulate; a_major: 0 K-major, 1 MN-major.
__device__ __forceinline__ constexpr uint32_t idesc_attn(uint32_t a_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (a_major << 15) | (static_cast<uint32_t>(NH >> 3) << 17) |
         (static_cast<uint32_t>(128 >> 4) << 24);
}

// Byte offset of element (row, k) in a [2 k-halves][16 rows][128 B] swizzled tile.
__device__ __forceinline__ uint32_t qp_offset(int row, int k) {
  const int half = k >> 6, kk = k & 63;
  const int chunk = kk >> 3;
  return half * (NH * 128) + row * 128 + ((chunk ^ (row & 7)) << 4) + (kk & 7) * 2;
}

__device__ __forceinline__ void named_sync_softmax() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

struct Item {
  int b, kvh, split, c0, c1, seq_len, tok0, tok1;
};

__device__ __forceinline__ Item decode_item(int idx, int Hkv, int S, int chunks_per_split, const int* seq_lens) {
  Item it;
  it.split = idx % S;
  it.kvh = (idx / S) % Hkv;
  it.b = idx / (S * Hkv);
  it.seq_len = seq_lens[it.b];
  const int nchunks = (it.seq_len + CHUNK - 1) / CHUNK;
  it.c0 = it.split * chunks_per_split;
  it.c1 = min(nchunks, it.c0 + chunks_per_split);
  it.tok0 = it.c0 * CHUNK;
  it.tok1 = min(it.seq_len, it.c1 * CHUNK);
  return it;
}

template <int G, int STAGES>
__device__ __forceinline__ void attn_body(const CUtensorMap* tmK, const CUtensorMap* tmV, const CUtensorMap* tmK16,
                                          const CUtensorMap* tmV16, const bf16* __restrict__ q,
                                          const int* __restrict__ block_tables, int max_blocks,
                                          const int* __restrict__ seq_lens, bf16* __restrict__ out,
                                          float* __restrict__ o_part, float* __restrict__ ml_part, int B, int Hkv,
                                          int S, int chunks_per_split, float scale_log2) {
  extern __shared__ uint8_t smem_raw[];
  Smem<STAGES>& sm = *reinterpret_cast<Smem<STAGES>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_items = B * Hkv * S;
  const int Hq = Hkv * G;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&sm.kfull[s], 1);
      mbar_init(&sm.vfull[s], 1);
      mbar_init(&sm.kempty[s], 1);
      mbar_init(&sm.vempty[s], 1);
    }
    mbar_init(&sm.s_full, 1);
    mbar_init(&sm.o_full, 1);
    mbar_init(&sm.s_empty, 4);
    mbar_init(&sm.p_full, 4);
    mbar_init(&sm.o_empty, 4);
    mbar_init(&sm.q_ready, 4);
    sm.abort = 0;
    fence_barrier_init();
    fence_proxy_async();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(tmK);
    tma_prefetch_desc(tmV);
    tma_prefetch_desc(tmK16);
    tma_prefetch_desc(tmV16);
  }
  if (warp == 1) {
    tmem_alloc(&sm.tmem, 32);
    tmem_relinquish();
  }
  // P rows for heads >= G stay zero for the whole kernel.
  for (int i = threadIdx.x; i < QP_BYTES / 16; i += blockDim.x) {
    reinterpret_cast<uint4*>(sm.p)[i] = make_uint4(0, 0, 0, 0);
    reinterpret_cast<uint4*>(sm.q)[i] = make_uint4(0, 0, 0, 0);
  }
  fence_proxy_async();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_trigger();
  pdl_wait();  // set-up above overlapped the previous kernel; its outputs (q, caches) are read below
  const uint32_t tmem = sm.tmem;
  const uint32_t t_s = tmem, t_o = tmem + NH;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int idx = blockIdx.x; idx < num_items && !*(volatile int*)&sm.abort; idx += gridDim.x) {
        const Item it = decode_item(idx, Hkv, S, chunks_per_split, seq_lens);
        const int* bt = block_tables + static_cast<size_t>(it.b) * max_blocks;
        // Only the live tokens of a chunk are read: whole pages, and the last
        // page in 16-token row blocks (a 16-row box at a 2 KB offset lands in
        // the same 128B-swizzled image as the rows of a full box). Rows not
        // loaded keep stale data: their scores are masked and their V rows
        // zeroed by the softmax warps before the PV MMA reads them.
        // The page ids of chunk c + 1 are read from the block table while
        // chunk c waits for its buffers, off the critical path.
        auto chunk_pages = [&](int c, int (&blocks)[2], int (&pages)[2]) {
          const int live = min(it.tok1, (c + 1) * CHUNK) - c * CHUNK;
#pragma unroll
          for (int pg = 0; pg < 2; ++pg) {
            const int n = min(max(live - pg * PAGE, 0), PAGE);
            blocks[pg] = (n + 15) / 16;  // 16-token blocks loaded (4 = the whole page)
            pages[pg] = blocks[pg] ? bt[2 * c + pg] : 0;
          }
        };
        int nblocks[2] = {0, 0}, npages[2] = {0, 0};
        if (it.c0 < it.c1) chunk_pages(it.c0, nblocks, npages);
        for (int c = it.c0; c < it.c1; ++c) {
          int blocks[2] = {nblocks[0], nblocks[1]};
          int rows[2];
#pragma unroll
          for (int pg = 0; pg < 2; ++pg) rows[pg] = (npages[pg] * Hkv + it.kvh) * PAGE;
          if (c + 1 < it.c1) chunk_pages(c + 1, nblocks, npages);
          const uint32_t bytes = static_cast<uint32_t>(blocks[0] + blocks[1]) * (2 * SUB_BYTES);  // K or V
          uint8_t* kbuf = sm.kv[stage];
#pragma unroll
          for (int kv = 0; kv < 2; ++kv) {  // K, then V
            uint64_t* empty = kv ? &sm.vempty[stage] : &sm.kempty[stage];
            uint64_t* full = kv ? &sm.vfull[stage] : &sm.kfull[stage];
            if (!mbar_wait(empty, phase ^ 1, FB_KERR_TIMEOUT_EMPTY)) {
              sm.abort = 1;
              continue;  // no copies for this chunk; the loop ends below
            }
            mbar_arrive_expect_tx(full, bytes);
            const CUtensorMap* whole = kv ? tmV : tmK;
            const CUtensorMap* part = kv ? tmV16 : tmK16;
            uint8_t* buf = kbuf + kv * KV_BYTES;
#pragma unroll
            for (int pg = 0; pg < 2; ++pg) {
              if (blocks[pg] == 0) continue;
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                uint8_t* dst = buf + h * HALF_STRIDE + pg * BOX_BYTES;
                if (blocks[pg] == 4) {
                  tma_load_2d(dst, whole, full, h * 64, rows[pg]);
                } else {
                  for (int j = 0; j < blocks[pg]; ++j)
                    tma_load_2d(dst + j * SUB_BYTES, part, full, h * 64, rows[pg] + 16 * j);
                }
              }
            }
          }
          if (*(volatile int*)&sm.abort) break;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // Drain: every issued load has been consumed (or the kernel aborted).
      for (int s = 0; s < STAGES; ++s) {
        mbar_wait(&sm.kempty[stage], phase ^ 1, FB_KERR_TIMEOUT_EMPTY);
        mbar_wait(&sm.vempty[stage], phase ^ 1, FB_KERR_TIMEOUT_EMPTY);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t id_qk = idesc_attn(0);
      constexpr uint32_t id_pv = idesc_attn(1);
      int stage = 0;
      uint32_t phase = 0;
      uint32_t cc = 0;  // chunks processed by this CTA
      uint32_t items_done = 0;
      bool ok = true;
      for (int idx = blockIdx.x; ok && idx < num_items && !*(volatile int*)&sm.abort; idx += gridDim.x) {
        const Item it = decode_item(idx, Hkv, S, chunks_per_split, seq_lens);
        if (it.c0 >= it.c1) continue;
        if (!mbar_wait(&sm.q_ready, items_done & 1, FB_KERR_TIMEOUT_FULL)) { ok = false; break; }
        ++items_done;
        for (int c = it.c0; c < it.c1; ++c, ++cc) {
          if (!mbar_wait(&sm.kfull[stage], phase, FB_KERR_TIMEOUT_FULL) ||
              !mbar_wait(&sm.s_empty, (cc & 1) ^ 1, FB_KERR_TIMEOUT_TMEM)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t kb = smem_u32(sm.kv[stage]);
          const uint32_t vb = kb + KV_BYTES;
          const uint32_t qb = smem_u32(sm.q);
          const uint32_t pb = smem_u32(sm.p);
#pragma unroll
          for (int j = 0; j < 8; ++j) {  // K = 128 head dims, 16 per MMA
            const uint32_t h = j >> 2, off = (j & 3) * 32;
            mma_bf16(t_s, desc_kmajor(kb + h * HALF_STRIDE + off), desc_kmajor(qb + h * (NH * 128) + off), id_qk,
                     j > 0 ? 1u : 0u);
          }
          mma_commit(&sm.s_full);
          mma_commit(&sm.kempty[stage]);  // K is free once QK completes
          if (!mbar_wait(&sm.p_full, cc & 1, FB_KERR_TIMEOUT_TMEM) ||
              !mbar_wait(&sm.o_empty, (cc & 1) ^ 1, FB_KERR_TIMEOUT_TMEM) ||
              !mbar_wait(&sm.vfull[stage], phase, FB_KERR_TIMEOUT_FULL)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int j = 0; j < 8; ++j) {  // K = 128 tokens, 16 per MMA
            const uint32_t h = j >> 2, off = (j & 3) * 32;
            mma_bf16(t_o, desc_mnmajor(vb + j * 2048, HALF_STRIDE, 1024), desc_kmajor(pb + h * (NH * 128) + off),
                     id_pv, j > 0 ? 1u : 0u);
          }
          mma_commit(&sm.o_full);
          mma_commit(&sm.vempty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) sm.abort = 1;
    }
  } else {
    // ---------------- softmax / epilogue (warps 2..5) ----------------
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // TMEM lane: token (for S) / head dim (for O)
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    uint32_t cc = 0;
    for (int idx = blockIdx.x; idx < num_items && !*(volatile int*)&sm.abort; idx += gridDim.x) {
      const Item it = decode_item(idx, Hkv, S, chunks_per_split, seq_lens);
      if (it.c0 >= it.c1) {
        if (S > 1 && r < G) {
          const size_t pidx = (static_cast<size_t>(it.b) * Hq + it.kvh * G + r) * S + it.split;
          ml_part[2 * pidx] = -INFINITY;
          ml_part[2 * pidx + 1] = 0.f;
        }
        continue;
      }
      // Q^T rows (heads) into the swizzled B tile: 16 rows x 16 chunks of 16 B.
      for (int e = r; e < G * 16; e += 128) {
        const int row = e >> 4, chunk = e & 15;
        const uint4 v = *reinterpret_cast<const uint4*>(
            q + (static_cast<size_t>(it.b) * Hq + it.kvh * G + row) * D + chunk * 8);
        *reinterpret_cast<uint4*>(sm.q + qp_offset(row, chunk * 8)) = v;
      }
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.q_ready);

      // The running max is the same in every softmax thread: kept in shared
      // memory (registers are the limit at three CTAs per SM). Chunk k reads
      // mrun[k & 1] and thread 0 writes the new max to mrun[(k + 1) & 1]
      // after the chunk's first barrier, so no read of a buffer overlaps its
      // next write.
      float l_thr[G], o[G];
#pragma unroll
      for (int g = 0; g < G; ++g) {
        if (r == 0) sm.mrun[cc & 1][g] = -INFINITY;
        l_thr[g] = 0.f;
        o[g] = 0.f;
      }
      for (int c = it.c0; c < it.c1; ++c, ++cc) {
        if (!mbar_wait(&sm.s_full, cc & 1, FB_KERR_TIMEOUT_TMEM)) {
          sm.abort = 1;
          break;
        }
        tc_fence_after();
        uint32_t sr[G];  // only the G head columns of S are live
        tmem_ld_cols<G>(t_s + lane_base, sr);
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.s_empty);
        const int tok = c * CHUNK + r;
        const bool valid = tok >= it.tok0 && tok < it.tok1;
        if (!valid) {
          // The PV MMA reads all 128 token rows of V: rows past the sequence
          // hold stale or never-written cache memory, and 0 * NaN = NaN, so
          // masked rows are zeroed here, after this chunk's V copies landed
          // (a 16-row tail box can cover tokens past the end).
          if (!mbar_wait(&sm.vfull[cc % STAGES], (cc / STAGES) & 1, FB_KERR_TIMEOUT_FULL)) sm.abort = 1;
          uint8_t* vrow = sm.kv[cc % STAGES] + KV_BYTES + r * 128;
#pragma unroll
          for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int i = 0; i < 8; ++i)
              reinterpret_cast<uint4*>(vrow + h * HALF_STRIDE)[i] = make_uint4(0, 0, 0, 0);
        }
        float s[G];
#pragma unroll
        for (int g = 0; g < G; ++g) {
          s[g] = valid ? __uint_as_float(sr[g]) * scale_log2 : -INFINITY;
          const float cmax = warp_max(s[g]);
          if (lane == 0) sm.red_max[quarter][g] = cmax;
        }
        named_sync_softmax();
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float mx = fmaxf(fmaxf(sm.red_max[0][g], sm.red_max[1][g]), fmaxf(sm.red_max[2][g], sm.red_max[3][g]));
          const float m_old = sm.mrun[cc & 1][g];
          const float m_new = fmaxf(m_old, mx);
          const float alpha = exp2f(m_old - m_new);
          // Kept in shared memory until the PV result arrives (registers are
          // the limit at three CTAs per SM); rewritten next chunk only after
          // every thread has passed that chunk's first barrier.
          if (r == 0) sm.alpha[g] = alpha;
          const float p = exp2f(s[g] - m_new);
          if (r == 0) sm.mrun[(cc + 1) & 1][g] = m_new;
          l_thr[g] = l_thr[g] * alpha + p;
          *reinterpret_cast<bf16*>(sm.p + qp_offset(g, r)) = f2bf(p);
        }
        fence_proxy_async();
        named_sync_softmax();  // red_max is rewritten next chunk
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.p_full);
        if (!mbar_wait(&sm.o_full, cc & 1, FB_KERR_TIMEOUT_TMEM)) {
          sm.abort = 1;
          break;
        }
        tc_fence_after();
        uint32_t orr[G];
        tmem_ld_cols<G>(t_o + lane_base, orr);
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.o_empty);
#pragma unroll
        for (int g = 0; g < G; ++g) o[g] = o[g] * sm.alpha[g] + __uint_as_float(orr[g]);
      }
      // l per head: sum over the 128 token lanes.
      float lsum[G];
#pragma unroll
      for (int g = 0; g < G; ++g) {
        lsum[g] = warp_sum(l_thr[g]);
      }
      if (lane == 0) {
#pragma unroll
        for (int g = 0; g < G; ++g) sm.red_l[quarter][g] = lsum[g];
      }
      named_sync_softmax();
#pragma unroll
      for (int g = 0; g < G; ++g) lsum[g] = sm.red_l[0][g] + sm.red_l[1][g] + sm.red_l[2][g] + sm.red_l[3][g];
      named_sync_softmax();
      // Thread r owns head dim r of every head.
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const int hq = it.kvh * G + g;
        if (S == 1) {
          out[(static_cast<size_t>(it.b) * Hq + hq) * D + r] = f2bf(o[g] / lsum[g]);
        } else {
          const size_t pidx = (static_cast<size_t>(it.b) * Hq + hq) * S + it.split;
          o_part[pidx * D + r] = o[g];
          if (r == 0) {
            ml_part[2 * pidx] = sm.mrun[cc & 1][g];  // written by this thread in the last chunk
            ml_part[2 * pidx + 1] = lsum[g];
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 32);
}

}  // namespace

#define FB_ATTN_TC_INSTANCE(G, ST, CTAS)                                                                         \
  extern "C" __global__ void __launch_bounds__(192, CTAS) fb_decode_attn_tc_g##G##_s##ST(                        \
      const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,                         \
      const __grid_constant__ CUtensorMap tmK16, const __grid_constant__ CUtensorMap tmV16, const bf16* q,       \
      const int* block_tables, int max_blocks, const int* seq_lens, bf16* out, float* o_part, float* ml_part,    \
      int B, int Hkv, int S, int chunks_per_split, float scale_log2) {                                            \
    attn_body<G, ST>(&tmK, &tmV, &tmK16, &tmV16, q, block_tables, max_blocks, seq_lens, out, o_part, ml_part, B, \
                     Hkv, S, chunks_per_split, scale_log2);                                                       \
  }

// 3-stage ring, one CTA per SM; or a single stage and three CTAs per SM.
FB_ATTN_TC_INSTANCE(4, 3, 1)
FB_ATTN_TC_INSTANCE(8, 3, 1)
FB_ATTN_TC_INSTANCE(4, 1, 3)
FB_ATTN_TC_INSTANCE(8, 1, 3)
