// Memory-bound kernels of the serving runner: weight init, embedding gather,
// RMSNorm, SiLU*mul, fused (QK-norm) + RoPE + paged KV-cache write, greedy
// argmax sampling, and small helpers. All use 16-byte vector accesses and one
// CTA (or warp) per row so each byte is read once.
#include "fb_common.cuh"

FB_DEFINE_STATUS

using namespace fbk;

// ---- deterministic random init ------------------------------------------------------
// Counter-based: value i depends only on (seed, i), so SAVE and LOAD processes
// (and any grid size) produce bit-identical weights. Normal via Box-Muller.
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  // splitmix64 finalizer (Steele, Lea, Flood 2014)
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

extern "C" __global__ void fb_init_normal_bf16(bf16* __restrict__ p, unsigned long long n, unsigned long long seed,
                                               float mean, float std) {
  pdl_entry();
  const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
  for (uint64_t pair = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; 2 * pair < n; pair += stride) {
    const uint64_t r = mix64(seed ^ mix64(pair));
    // 24-bit uniforms in (0, 1]
    const float u1 = (static_cast<float>((r >> 40) & 0xFFFFFF) + 1.0f) * (1.0f / 16777216.0f);
    const float u2 = static_cast<float>((r >> 16) & 0xFFFFFF) * (1.0f / 16777216.0f);
    const float rad = sqrtf(-2.0f * logf(u1));
    float s, c;
    sincosf(6.283185307179586f * u2, &s, &c);
    const uint64_t i = 2 * pair;
    p[i] = f2bf(mean + std * rad * c);
    if (i + 1 < n) p[i + 1] = f2bf(mean + std * rad * s);
  }
}

extern "C" __global__ void fb_fill_bf16(bf16* __restrict__ p, unsigned long long n, float v) {
  pdl_entry();
  const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
  const bf16 b = f2bf(v);
  for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < n; i += stride) p[i] = b;
}

// ---- embedding ----------------------------------------------------------------------
// out[t, :] = table[ids[t], :]; H % 8 == 0.
extern "C" __global__ void fb_embedding(const int* __restrict__ ids, const bf16* __restrict__ table,
                                        bf16* __restrict__ out, int T, int H, int vocab) {
  pdl_entry();
  const int t = blockIdx.x;
  if (t >= T) return;
  int id = ids[t];
  if (id < 0 || id >= vocab) {
    set_status(FB_KERR_BAD_ARG);
    id = 0;
  }
  const uint4* src = reinterpret_cast<const uint4*>(table + static_cast<size_t>(id) * H);
  uint4* dst = reinterpret_cast<uint4*>(out + static_cast<size_t>(t) * H);
  for (int i = threadIdx.x; i < H / 8; i += blockDim.x) dst[i] = __ldg(src + i);
}

// ---- RMSNorm ------------------------------------------------------------------------
// out[t] = x[t] * rsqrt(mean(x[t]^2) + eps) * w. One CTA per row, 16-byte loads,
// row kept in registers (H <= 8 * 8 * blockDim).
template <int VPT>
__device__ __forceinline__ void rmsnorm_row(const bf16* __restrict__ x, const bf16* __restrict__ w,
                                            bf16* __restrict__ out, int H, float eps) {
  __shared__ float red[32];
  const int nv = H / 8;
  float v[VPT][8];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int i = threadIdx.x + k * blockDim.x;
    if (i < nv) {
      unpack8(reinterpret_cast<const uint4*>(x)[i], v[k]);
#pragma unroll
      for (int e = 0; e < 8; ++e) ss += v[k][e] * v[k][e];
    }
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float s = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    s = warp_sum(s);
    if (threadIdx.x == 0) red[0] = s;
  }
  __syncthreads();
  const float inv = rsqrtf(red[0] / static_cast<float>(H) + eps);
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int i = threadIdx.x + k * blockDim.x;
    if (i < nv) {
      float wf[8], o[8];
      unpack8(reinterpret_cast<const uint4*>(w)[i], wf);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = v[k][e] * inv * wf[e];
      reinterpret_cast<uint4*>(out)[i] = pack8(o);
    }
  }
}

extern "C" __global__ void __launch_bounds__(256) fb_rmsnorm(const bf16* __restrict__ x, const bf16* __restrict__ w,
                                                              bf16* __restrict__ out, int T, int H, float eps) {
  pdl_entry();
  const int t = blockIdx.x;
  if (t >= T) return;
  if (H > 8 * 256 * 8) {
    set_status(FB_KERR_BAD_ARG);
    return;
  }
  rmsnorm_row<8>(x + static_cast<size_t>(t) * H, w, out + static_cast<size_t>(t) * H, H, eps);
}

// Residual add of split-K GEMM slices fused with the next RMSNorm:
//   h[t] = bf16(sum_s part[s][t] + h[t]);  x[t] = rmsnorm(h[t]) * w
// (sum in split order, then the residual: the same arithmetic as the GEMM's
// own residual epilogue, so split and unsplit GEMMs round the same way).
extern "C" __global__ void __launch_bounds__(256) fb_add_rmsnorm_partials(
    const float* __restrict__ part, int S, long long stride, bf16* __restrict__ h, const bf16* __restrict__ w,
    bf16* __restrict__ x, int T, int H, float eps) {
  pdl_entry();
  constexpr int VPT = 4;  // H <= 256 threads * 4 vectors * 8
  __shared__ float red[32];
  const int t = blockIdx.x;
  if (t >= T) return;
  if (H > 256 * VPT * 8) {
    set_status(FB_KERR_BAD_ARG);
    return;
  }
  const int nv = H / 8;
  bf16* hrow = h + static_cast<size_t>(t) * H;
  float v[VPT][8];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int i = threadIdx.x + k * blockDim.x;
    if (i >= nv) continue;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int s = 0; s < S; ++s) {
      const float4* p = reinterpret_cast<const float4*>(part + s * stride + static_cast<size_t>(t) * H + i * 8);
      const float4 a = __ldcs(p), b = __ldcs(p + 1);
      acc[0] += a.x; acc[1] += a.y; acc[2] += a.z; acc[3] += a.w;
      acc[4] += b.x; acc[5] += b.y; acc[6] += b.z; acc[7] += b.w;
    }
    float r[8];
    unpack8(reinterpret_cast<const uint4*>(hrow)[i], r);
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] += r[e];
    const uint4 packed = pack8(acc);
    reinterpret_cast<uint4*>(hrow)[i] = packed;
    unpack8(packed, v[k]);  // normalise the rounded value, as the unsplit path does
#pragma unroll
    for (int e = 0; e < 8; ++e) ss += v[k][e] * v[k][e];
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float s = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    s = warp_sum(s);
    if (threadIdx.x == 0) red[0] = s;
  }
  __syncthreads();
  const float inv = rsqrtf(red[0] / static_cast<float>(H) + eps);
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int i = threadIdx.x + k * blockDim.x;
    if (i >= nv) continue;
    float wf[8], o[8];
    unpack8(reinterpret_cast<const uint4*>(w)[i], wf);
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = v[k][e] * inv * wf[e];
    reinterpret_cast<uint4*>(x + static_cast<size_t>(t) * H)[i] = pack8(o);
  }
}

// ---- SiLU * mul ---------------------------------------------------------------------
// gu[t] = [gate (I) | up (I)]; out[t, i] = silu(gate) * up.
extern "C" __global__ void fb_silu_mul(const bf16* __restrict__ gu, bf16* __restrict__ out, int T, int I) {
  pdl_entry();
  const int nv = I / 8;
  const uint64_t total = static_cast<uint64_t>(T) * nv;
  for (uint64_t k = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; k < total;
       k += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    const int t = static_cast<int>(k / nv), i = static_cast<int>(k % nv);
    const uint4* row = reinterpret_cast<const uint4*>(gu + static_cast<size_t>(t) * 2 * I);
    float g[8], u[8], o[8];
    unpack8(row[i], g);
    unpack8(row[nv + i], u);
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = g[e] / (1.0f + __expf(-g[e])) * u[e];
    reinterpret_cast<uint4*>(out + static_cast<size_t>(t) * I)[i] = pack8(o);
  }
}

// ---- (QK-norm +) RoPE + paged KV write ------------------------------------------------
// qkv[t] = [q heads (Hq*128) | k heads (Hkv*128) | v heads (Hkv*128)].
// One warp per head; lane l holds dims [4l, 4l+4). RoPE is the half-rotation
// form (dim i pairs with i+64) with a precomputed fp32 (cos, sin) table
// [max_pos, 64]. K/V go to the paged cache [blocks, Hkv, page, 128] at
// slot_mapping[t] (negative slot = padding token, not written). If k_out /
// v_out are non-null the rotated K and the V heads are also written packed to
// [T, Hkv, 128] (prefill attention reads them from there). With S > 0 the
// input is the S fp32 split-K slices of the QKV GEMM ([S][T][ld_qkv], summed
// here in split order) instead of the bf16 qkv matrix.
extern "C" __global__ void __launch_bounds__(256) fb_rope_kv_write(
    const bf16* __restrict__ qkv, int ld_qkv, const int* __restrict__ positions, const float2* __restrict__ cos_sin,
    const bf16* __restrict__ q_norm_w, const bf16* __restrict__ k_norm_w, float eps, int use_qk_norm,
    bf16* __restrict__ q_out, bf16* __restrict__ k_cache, bf16* __restrict__ v_cache, const int* __restrict__ slots,
    int T, int Hq, int Hkv, int page, bf16* __restrict__ k_out, bf16* __restrict__ v_out,
    const float* __restrict__ part, int S, long long part_stride) {
  pdl_entry();
  const int t = blockIdx.x;
  const int h = blockIdx.y * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= T || h >= Hq + 2 * Hkv) return;
  const size_t col = static_cast<size_t>(t) * ld_qkv + h * 128 + lane * 4;
  float x[4];
  if (S > 0) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s = 0; s < S; ++s) {
      const float4 p = __ldcs(reinterpret_cast<const float4*>(part + s * part_stride + col));
      acc.x += p.x;
      acc.y += p.y;
      acc.z += p.z;
      acc.w += p.w;
    }
    // Round through bf16 like the unsplit GEMM epilogue does.
    x[0] = bf2f(f2bf(acc.x));
    x[1] = bf2f(f2bf(acc.y));
    x[2] = bf2f(f2bf(acc.z));
    x[3] = bf2f(f2bf(acc.w));
  } else {
    const uint2 raw = *reinterpret_cast<const uint2*>(qkv + col);
    const float2 a = __bfloat1622float2(*reinterpret_cast<const bf162*>(&raw.x));
    const float2 b = __bfloat1622float2(*reinterpret_cast<const bf162*>(&raw.y));
    x[0] = a.x;
    x[1] = a.y;
    x[2] = b.x;
    x[3] = b.y;
  }
  const bool is_v = h >= Hq + Hkv;
  if (!is_v) {
    if (use_qk_norm) {
      float ss = x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3];
      ss = warp_sum(ss);
      const float inv = rsqrtf(ss * (1.0f / 128.0f) + eps);
      const bf16* w = (h < Hq ? q_norm_w : k_norm_w) + lane * 4;
#pragma unroll
      for (int e = 0; e < 4; ++e) x[e] = x[e] * inv * bf2f(w[e]);
    }
    float p[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) p[e] = __shfl_xor_sync(0xffffffffu, x[e], 16);
    const int pos = positions[t];
    const float2* cs = cos_sin + static_cast<size_t>(pos) * 64 + (lane & 15) * 4;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 c = cs[e];
      x[e] = lane < 16 ? x[e] * c.x - p[e] * c.y : x[e] * c.x + p[e] * c.y;
    }
  }
  uint2 o;
  *reinterpret_cast<bf162*>(&o.x) = __floats2bfloat162_rn(x[0], x[1]);
  *reinterpret_cast<bf162*>(&o.y) = __floats2bfloat162_rn(x[2], x[3]);
  if (h < Hq) {
    *reinterpret_cast<uint2*>(q_out + (static_cast<size_t>(t) * Hq + h) * 128 + lane * 4) = o;
    return;
  }
  const int kvh = is_v ? h - Hq - Hkv : h - Hq;
  bf16* packed = is_v ? v_out : k_out;
  if (packed) *reinterpret_cast<uint2*>(packed + (static_cast<size_t>(t) * Hkv + kvh) * 128 + lane * 4) = o;
  const int slot = slots[t];
  if (slot < 0) return;
  const size_t blk = static_cast<size_t>(slot / page), off = static_cast<size_t>(slot % page);
  bf16* dst = (is_v ? v_cache : k_cache) + ((blk * Hkv + kvh) * page + off) * 128 + lane * 4;
  *reinterpret_cast<uint2*>(dst) = o;
}

// ---- greedy sampling ------------------------------------------------------------------
// out[t] = argmax_v logits[t, v] (lowest index on ties). One CTA per row.
extern "C" __global__ void __launch_bounds__(512) fb_argmax(const bf16* __restrict__ logits, int* __restrict__ out,
                                                             int T, int V, long long ld) {
  pdl_entry();
  const int t = blockIdx.x;
  if (t >= T) return;
  const bf16* row = logits + static_cast<size_t>(t) * ld;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  const int nv = V / 8;
  for (int i = threadIdx.x; i < nv; i += blockDim.x) {
    float f[8];
    unpack8(reinterpret_cast<const uint4*>(row)[i], f);
#pragma unroll
    for (int e = 0; e < 8; ++e)
      if (f[e] > best) {
        best = f[e];
        bi = i * 8 + e;
      }
  }
  for (int i = nv * 8 + threadIdx.x; i < V; i += blockDim.x) {
    const float f = bf2f(row[i]);
    if (f > best) {
      best = f;
      bi = i;
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
  __shared__ float sb[16];
  __shared__ int si[16];
  if ((threadIdx.x & 31) == 0) {
    sb[threadIdx.x >> 5] = best;
    si[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w)
      if (sb[w] > best || (sb[w] == best && si[w] < bi)) {
        best = sb[w];
        bi = si[w];
      }
    out[t] = bi;
  }
}

// ---- decode-step bookkeeping ----------------------------------------------------------
// For each sequence b of a decode batch: position = seq_len (before the new
// token), new slot from the block table, seq_len += 1. Runs inside the decode
// graph so a captured graph can be replayed step after step with no host work
// except copying in the sampled tokens.
extern "C" __global__ void fb_decode_advance(int* __restrict__ seq_lens, int* __restrict__ positions,
                                             int* __restrict__ slots, const int* __restrict__ block_tables,
                                             int max_blocks, int page, int B, const int* __restrict__ active) {
  pdl_entry();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  if (active && !active[b]) {
    positions[b] = 0;
    slots[b] = -1;
    return;
  }
  const int pos = seq_lens[b];
  positions[b] = pos;
  const int blk = block_tables[static_cast<size_t>(b) * max_blocks + pos / page];
  slots[b] = blk * page + pos % page;
  seq_lens[b] = pos + 1;
}

// Copies next-step input ids from the sampled tokens (device-side feedback).
extern "C" __global__ void fb_copy_i32(const int* __restrict__ src, int* __restrict__ dst, int n) {
  pdl_entry();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) dst[i] = src[i];
}
