// Attention kernels for the serving runner (head_dim 128, bf16, GQA).
//
// fb_decode_attn_g{4,8}: paged decode attention, one query token per
//   sequence, split-KV ("flash-decoding"). CTA = (split, kv head, sequence);
//   the G query heads of a KV head share every K/V byte read, so each KV byte
//   is read from HBM exactly once per step. K/V pages (64 tokens x 128 dims,
//   16 KB each, contiguous per (block, kv head)) stream through a
//   double-buffered cp.async ring; scores and softmax are fp32 in the log2
//   domain. With one split the CTA writes the bf16 output; otherwise fp32
//   partials (o, m, l) go to a workspace merged by fb_decode_attn_combine.
//   The grid covers the longest possible context so the launch shape is fixed
//   inside CUDA graphs; splits past a sequence's length exit immediately.
//
// fb_prefill_attn: causal attention over a packed batch of prompts
//   (cu_seqlens), one CTA per (64-query tile, head), K/V tiles in shared
//   memory, online softmax.
#include "fb_common.cuh"

FB_DEFINE_STATUS

using namespace fbk;

namespace {

constexpr int D = 128;
constexpr int PAGE = 64;

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Copy one 16 KB page (64 x 128 bf16) with 128 threads.
__device__ __forceinline__ void load_page(bf16* dst, const bf16* src) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int c = threadIdx.x + i * 128;
    cp_async16(dst + c * 8, src + c * 8);
  }
}

template <int G>
__device__ __forceinline__ void decode_attn(const bf16* __restrict__ q, const bf16* __restrict__ k_cache,
                                            const bf16* __restrict__ v_cache, const int* __restrict__ block_tables,
                                            int max_blocks, const int* __restrict__ seq_lens, bf16* __restrict__ out,
                                            float* __restrict__ o_part, float* __restrict__ ml_part, int Hkv,
                                            int pages_per_split, float scale_log2) {
  extern __shared__ __align__(16) uint8_t smem[];
  bf16* kbuf = reinterpret_cast<bf16*>(smem);              // [2][64][128]
  bf16* vbuf = kbuf + 2 * PAGE * D;                         // [2][64][128]
  float* s_s = reinterpret_cast<float*>(vbuf + 2 * PAGE * D);  // [G][64]
  float* p_s = s_s + G * PAGE;                              // [64][G]
  float* alpha_s = p_s + PAGE * G;                          // [G]
  float* red = alpha_s + G;                                 // [G][128]

  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int S = gridDim.x;
  const int Hq = Hkv * G;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int seq_len = seq_lens[b];
  const int num_pages = (seq_len + PAGE - 1) / PAGE;
  const int p0 = split * pages_per_split;
  const int p1 = min(num_pages, p0 + pages_per_split);

  if (p0 >= p1) {
    if (S > 1 && tid < G) {
      const size_t idx = (static_cast<size_t>(b) * Hq + kvh * G + tid) * S + split;
      ml_part[2 * idx] = -INFINITY;
      ml_part[2 * idx + 1] = 0.f;
    }
    return;
  }

  // q slice in registers: dims [c*8, c*8+8) and [64+c*8, 64+c*8+8), pre-scaled.
  const int c = tid & 7, j0 = tid >> 3;
  float qr[G][16];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const bf16* qp = q + (static_cast<size_t>(b) * Hq + kvh * G + g) * D;
    float a[8], bb[8];
    unpack8(*reinterpret_cast<const uint4*>(qp + c * 8), a);
    unpack8(*reinterpret_cast<const uint4*>(qp + 64 + c * 8), bb);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      qr[g][e] = a[e] * scale_log2;
      qr[g][8 + e] = bb[e] * scale_log2;
    }
  }

  // PV ownership: dims d0, d0+1; token half th.
  const int d0 = 2 * (tid & 63), th = tid >> 6;
  float o[G][2];
#pragma unroll
  for (int g = 0; g < G; ++g) o[g][0] = o[g][1] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};  // heads warp, warp+4

  const int* bt = block_tables + static_cast<size_t>(b) * max_blocks;
  auto page_ptr = [&](const bf16* cache, int p) {
    return cache + (static_cast<size_t>(bt[p]) * Hkv + kvh) * (PAGE * D);
  };
  load_page(kbuf, page_ptr(k_cache, p0));
  load_page(vbuf, page_ptr(v_cache, p0));
  cp_async_commit();

  for (int p = p0; p < p1; ++p) {
    const int buf = (p - p0) & 1;
    if (p + 1 < p1) {
      load_page(kbuf + (buf ^ 1) * PAGE * D, page_ptr(k_cache, p + 1));
      load_page(vbuf + (buf ^ 1) * PAGE * D, page_ptr(v_cache, p + 1));
    }
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const bf16* kt = kbuf + buf * PAGE * D;
    const bf16* vt = vbuf + buf * PAGE * D;
    const int valid = min(PAGE, seq_len - p * PAGE);

    // ---- scores: s[g][j] = q_g . k_j (log2 domain) ----
#pragma unroll
    for (int pass = 0; pass < 4; ++pass) {
      const int j = j0 + pass * 16;
      float kf[16];
      unpack8(*reinterpret_cast<const uint4*>(kt + j * D + c * 8), *reinterpret_cast<float(*)[8]>(kf));
      unpack8(*reinterpret_cast<const uint4*>(kt + j * D + 64 + c * 8), *reinterpret_cast<float(*)[8]>(kf + 8));
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float acc = 0.f;
#pragma unroll
        for (int e = 0; e < 16; ++e) acc = fmaf(qr[g][e], kf[e], acc);
        acc += __shfl_xor_sync(0xffffffffu, acc, 1);
        acc += __shfl_xor_sync(0xffffffffu, acc, 2);
        acc += __shfl_xor_sync(0xffffffffu, acc, 4);
        if (c == (g & 7)) s_s[g * PAGE + j] = acc;
      }
    }
    __syncthreads();

    // ---- online softmax: warp w owns heads w and w+4 ----
#pragma unroll
    for (int hh = 0; hh < (G + 3) / 4; ++hh) {
      const int g = warp + hh * 4;
      if (g < G) {
        const float sa = lane < valid ? s_s[g * PAGE + lane] : -INFINITY;
        const float sb = lane + 32 < valid ? s_s[g * PAGE + lane + 32] : -INFINITY;
        const float tmax = warp_max(fmaxf(sa, sb));
        const float m_new = fmaxf(m_run[hh], tmax);
        const float pa = exp2f(sa - m_new), pb = exp2f(sb - m_new);
        const float alpha = exp2f(m_run[hh] - m_new);
        l_run[hh] = l_run[hh] * alpha + warp_sum(pa + pb);
        m_run[hh] = m_new;
        p_s[lane * G + g] = pa;
        p_s[(lane + 32) * G + g] = pb;
        if (lane == 0) alpha_s[g] = alpha;
      }
    }
    __syncthreads();

    // ---- o = o * alpha + P V ----
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float a = alpha_s[g];
      o[g][0] *= a;
      o[g][1] *= a;
    }
    const int jb = th * 32, je = min(jb + 32, valid);
    for (int j = jb; j < je; ++j) {
      const float2 v = __bfloat1622float2(*reinterpret_cast<const bf162*>(vt + j * D + d0));
      float pj[G];
      if constexpr (G % 4 == 0) {
#pragma unroll
        for (int g4 = 0; g4 < G / 4; ++g4) {
          const float4 pv = *reinterpret_cast<const float4*>(p_s + j * G + g4 * 4);
          pj[g4 * 4] = pv.x;
          pj[g4 * 4 + 1] = pv.y;
          pj[g4 * 4 + 2] = pv.z;
          pj[g4 * 4 + 3] = pv.w;
        }
      } else {
#pragma unroll
        for (int g = 0; g < G; ++g) pj[g] = p_s[j * G + g];
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
        o[g][0] = fmaf(pj[g], v.x, o[g][0]);
        o[g][1] = fmaf(pj[g], v.y, o[g][1]);
      }
    }
    __syncthreads();  // buffers and p_s are rewritten next iteration
  }

  // ---- merge the two token halves ----
  if (th == 1) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      red[g * D + d0] = o[g][0];
      red[g * D + d0 + 1] = o[g][1];
    }
  }
  // publish per-head (m, l): the owning warp's lane 0
  float* ml_s = s_s;  // reuse: [G][2]
  if (lane == 0) {
#pragma unroll
    for (int hh = 0; hh < (G + 3) / 4; ++hh) {
      const int g = warp + hh * 4;
      if (g < G) {
        ml_s[2 * g] = m_run[hh];
        ml_s[2 * g + 1] = l_run[hh];
      }
    }
  }
  __syncthreads();
  if (th == 0) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float x0 = o[g][0] + red[g * D + d0];
      const float x1 = o[g][1] + red[g * D + d0 + 1];
      const int hq = kvh * G + g;
      if (S == 1) {
        const float inv = 1.0f / ml_s[2 * g + 1];
        *reinterpret_cast<bf162*>(out + (static_cast<size_t>(b) * Hq + hq) * D + d0) =
            __floats2bfloat162_rn(x0 * inv, x1 * inv);
      } else {
        const size_t idx = (static_cast<size_t>(b) * Hq + hq) * S + split;
        *reinterpret_cast<float2*>(o_part + idx * D + d0) = make_float2(x0, x1);
        if (d0 == 0) {
          ml_part[2 * idx] = ml_s[2 * g];
          ml_part[2 * idx + 1] = ml_s[2 * g + 1];
        }
      }
    }
  }
}

}  // namespace

#define FB_DECODE_INSTANCE(G)                                                                                     \
  extern "C" __global__ void __launch_bounds__(128) fb_decode_attn_g##G(                                          \
      const bf16* q, const bf16* k_cache, const bf16* v_cache, const int* block_tables, int max_blocks,           \
      const int* seq_lens, bf16* out, float* o_part, float* ml_part, int Hkv, int pages_per_split,                \
      float scale_log2) {                                                                                          \
    pdl_entry();                                                                                                   \
    decode_attn<G>(q, k_cache, v_cache, block_tables, max_blocks, seq_lens, out, o_part, ml_part, Hkv,           \
                   pages_per_split, scale_log2);                                                                   \
  }

FB_DECODE_INSTANCE(4)
FB_DECODE_INSTANCE(8)

// Merge split partials: one CTA per (sequence, query head), one thread per dim.
extern "C" __global__ void __launch_bounds__(128) fb_decode_attn_combine(const float* __restrict__ o_part,
                                                                          const float* __restrict__ ml_part,
                                                                          bf16* __restrict__ out, int Hq, int S) {
  pdl_entry();
  const int b = blockIdx.x, h = blockIdx.y, d = threadIdx.x;
  const size_t base = (static_cast<size_t>(b) * Hq + h) * S;
  float M = -INFINITY;
  for (int s = 0; s < S; ++s) M = fmaxf(M, ml_part[2 * (base + s)]);
  float L = 0.f, acc = 0.f;
  for (int s = 0; s < S; ++s) {
    const float m = ml_part[2 * (base + s)];
    if (m == -INFINITY) continue;
    const float w = exp2f(m - M);
    L += ml_part[2 * (base + s) + 1] * w;
    acc += o_part[(base + s) * D + d] * w;
  }
  out[(static_cast<size_t>(b) * Hq + h) * D + d] = f2bf(L > 0.f ? acc / L : 0.f);
}

// ---- prefill (causal) ------------------------------------------------------------------
// q: [T, Hq, 128], k/v: [T, Hkv, 128] (packed prompts, cu_seqlens[B+1]).
// CTA = (query tile of 64 rows, q head); 128 threads: thread t owns query row
// t>>1 and head-dim half (t&1). Scores for a 64-key tile are accumulated in
// registers (64 per thread), then P.V with the thread's 64 output dims.
constexpr int PQ = 64, PK = 32;

extern "C" __global__ void __launch_bounds__(128) fb_prefill_attn(
    const bf16* __restrict__ q, const bf16* __restrict__ k, const bf16* __restrict__ v, int ld_q, int ld_k, int ld_v,
    bf16* __restrict__ out, int ld_o, const int* __restrict__ cu_seqlens, const int* __restrict__ tile_seq,
    const int* __restrict__ tile_start, int Hq, int Hkv, float scale_log2) {
  pdl_entry();
  __shared__ __align__(16) bf16 ks[PK][D + 8];
  __shared__ __align__(16) bf16 vs[PK][D + 8];
  const int tile = blockIdx.x, h = blockIdx.y;
  const int seq = tile_seq[tile];
  const int q0 = tile_start[tile];  // first query index within the sequence
  const int base = cu_seqlens[seq];
  const int len = cu_seqlens[seq + 1] - base;
  const int kvh = h / (Hq / Hkv);
  const int r = threadIdx.x >> 1, half = threadIdx.x & 1;
  const int qi = q0 + r;
  const bool valid_q = qi < len;

  float qv[64];
  {
    const bf16* qp = q + static_cast<size_t>(base + min(qi, len - 1)) * ld_q + h * D + half * 64;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float f[8];
      unpack8(*reinterpret_cast<const uint4*>(qp + i * 8), f);
#pragma unroll
      for (int e = 0; e < 8; ++e) qv[i * 8 + e] = f[e] * scale_log2;
    }
  }
  float acc[64];
#pragma unroll
  for (int i = 0; i < 64; ++i) acc[i] = 0.f;
  float m = -INFINITY, l = 0.f;
  const int kend = min(len, q0 + PQ);  // causal: keys <= last query of the tile
  for (int k0 = 0; k0 < kend; k0 += PK) {
    __syncthreads();
    for (int i = threadIdx.x; i < PK * (D / 8); i += 128) {
      const int row = i / (D / 8), col = (i % (D / 8)) * 8;
      const int kj = min(k0 + row, len - 1);
      *reinterpret_cast<uint4*>(&ks[row][col]) =
          *reinterpret_cast<const uint4*>(k + static_cast<size_t>(base + kj) * ld_k + kvh * D + col);
      *reinterpret_cast<uint4*>(&vs[row][col]) =
          *reinterpret_cast<const uint4*>(v + static_cast<size_t>(base + kj) * ld_v + kvh * D + col);
    }
    __syncthreads();
    float s[PK];
#pragma unroll
    for (int j = 0; j < PK; ++j) {
      float a = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float f[8];
        unpack8(*reinterpret_cast<const uint4*>(&ks[j][half * 64 + i * 8]), f);
#pragma unroll
        for (int e = 0; e < 8; ++e) a = fmaf(qv[i * 8 + e], f[e], a);
      }
      a += __shfl_xor_sync(0xffffffffu, a, 1);
      s[j] = (k0 + j <= qi && k0 + j < len) ? a : -INFINITY;
    }
    float tmax = -INFINITY;
#pragma unroll
    for (int j = 0; j < PK; ++j) tmax = fmaxf(tmax, s[j]);
    const float m_new = fmaxf(m, tmax);
    const float alpha = m_new == -INFINITY ? 1.f : exp2f(m - m_new);
    float psum = 0.f;
#pragma unroll
    for (int j = 0; j < PK; ++j) {
      s[j] = m_new == -INFINITY ? 0.f : exp2f(s[j] - m_new);
      psum += s[j];
    }
    l = l * alpha + psum;
    m = m_new;
#pragma unroll
    for (int i = 0; i < 64; ++i) acc[i] *= alpha;
#pragma unroll
    for (int j = 0; j < PK; ++j) {
      const float pj = s[j];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float f[8];
        unpack8(*reinterpret_cast<const uint4*>(&vs[j][half * 64 + i * 8]), f);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[i * 8 + e] = fmaf(pj, f[e], acc[i * 8 + e]);
      }
    }
  }
  if (!valid_q) return;
  const float inv = l > 0.f ? 1.f / l : 0.f;
  bf16* op = out + static_cast<size_t>(base + qi) * ld_o + h * D + half * 64;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float f[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) f[e] = acc[i * 8 + e] * inv;
    *reinterpret_cast<uint4*>(op + i * 8) = pack8(f);
  }
}
