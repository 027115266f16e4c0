// Collectives over NVLink 5 / NVSwitch between ranks (one process per GPU)
// whose symmetric buffers are mapped at identical virtual addresses in every
// process: rank r's buffer is at base + r * stride (peer memory via P2P), and
// the NVLS multicast object of the same buffers at mc_base (one store or
// ld_reduce reaches every GPU through the switch).
//
// Control block at the start of every rank's buffer:
//   [FLAG_OFF + 4*src]  epoch last signalled by rank src to this rank
//   [EPOCH_OFF]         this rank's own barrier epoch counter
// Every wait is bounded (FB_WAIT_NS); on expiry the kernel records
// FB_KERR_TIMEOUT_PEER in fb_status and returns instead of hanging.
//
// Kernels:
//   fb_sym_barrier            all ranks arrive; release/acquire at system scope
//   fb_allreduce_oneshot_bf16 sum of all ranks' buffers, read over P2P in rank
//                             order (deterministic), written locally
//   fb_allreduce_nvls_bf16    each rank reduces a 1/world shard with
//                             multimem.ld_reduce (fp32 accumulation in the
//                             switch) and multicasts it back (multimem.st)
//   fb_add_rmsnorm_slots      h += sum over ranks of their output slots (rank
//                             order), then RMSNorm: the consumer half of the
//                             fused GEMM -> all-reduce (the GEMM epilogue
//                             multicasts each rank's tile into slot[rank])
//   fb_argmax_shard/combine   greedy sampling over a vocab-sharded lm_head
#include "fb_common.cuh"

FB_DEFINE_STATUS

using namespace fbk;

namespace {
constexpr int FLAG_OFF = 0;
constexpr int EPOCH_OFF = 512;

__device__ __forceinline__ void st_release_sys(uint64_t addr, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(uint64_t addr) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
  return v;
}
}  // namespace

extern "C" __global__ void __launch_bounds__(64) fb_sym_barrier(unsigned long long base,
                                                                 unsigned long long stride, int rank, int world) {
  pdl_entry();
  __shared__ uint32_t epoch;
  const int t = threadIdx.x;
  if (t == 0) {
    uint32_t* ctr = reinterpret_cast<uint32_t*>(base + rank * stride + EPOCH_OFF);
    epoch = *ctr + 1;
    *ctr = epoch;
  }
  __syncthreads();
  const uint32_t e = epoch;
  if (t < world) {
    // Release: everything this GPU wrote before (earlier kernels of the stream
    // included) is visible to rank t before it sees the new epoch.
    st_release_sys(base + t * stride + FLAG_OFF + 4ull * rank, e);
    const uint64_t mine = base + rank * stride + FLAG_OFF + 4ull * t;
    const uint64_t t0 = globaltimer();
    uint32_t it = 0;
    while (static_cast<int32_t>(ld_acquire_sys(mine) - e) < 0) {
      if ((++it & 1023u) == 0 && globaltimer() - t0 > FB_WAIT_NS) {
        set_status(FB_KERR_TIMEOUT_PEER);
        break;
      }
    }
  }
  __syncthreads();
}

extern "C" __global__ void fb_allreduce_oneshot_bf16(unsigned long long base, unsigned long long stride,
                                                     unsigned long long offset, bf16* __restrict__ out,
                                                     long long n, int world) {
  pdl_entry();
  const long long nv = n / 8;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < nv;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int r = 0; r < world; ++r) {
      const uint4 v = __ldcv(reinterpret_cast<const uint4*>(base + r * stride + offset) + i);
      float f[8];
      unpack8(v, f);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] += f[e];
    }
    reinterpret_cast<uint4*>(out)[i] = pack8(acc);
  }
}

extern "C" __global__ void fb_allreduce_nvls_bf16(unsigned long long mc_in, unsigned long long mc_out,
                                                  long long n, int rank, int world) {
  pdl_entry();
  const long long nv = n / 8;
  const long long per = (nv + world - 1) / world;
  const long long lo = rank * per, hi = min(nv, lo + per);
  for (long long i = lo + blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < hi;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    uint32_t a, b, c, d;
    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0,%1,%2,%3}, [%4];"
                 : "=r"(a), "=r"(b), "=r"(c), "=r"(d)
                 : "l"(mc_in + i * 16)
                 : "memory");
    asm volatile("multimem.st.relaxed.sys.global.v4.bf16x2 [%0], {%1,%2,%3,%4};" ::"l"(mc_out + i * 16), "r"(a),
                 "r"(b), "r"(c), "r"(d)
                 : "memory");
  }
}

// h[t] = bf16(sum_r slot[r][t] + h[t]); x[t] = rmsnorm(h[t]) * w.
extern "C" __global__ void __launch_bounds__(256) fb_add_rmsnorm_slots(
    const bf16* __restrict__ slots, int W, long long slot_stride, bf16* __restrict__ h,
    const bf16* __restrict__ w, bf16* __restrict__ x, int T, int H, float eps) {
  pdl_entry();
  constexpr int VPT = 4;
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
    for (int r = 0; r < W; ++r) {
      float f[8];
      unpack8(__ldcv(reinterpret_cast<const uint4*>(slots + r * slot_stride + static_cast<size_t>(t) * H) + i), f);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] += f[e];
    }
    float hv[8];
    unpack8(reinterpret_cast<const uint4*>(hrow)[i], hv);
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] += hv[e];
    const uint4 packed = pack8(acc);
    reinterpret_cast<uint4*>(hrow)[i] = packed;
    unpack8(packed, v[k]);
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

// Local argmax of a vocab shard; the (value, global index) pair of each row is
// stored to pairs[rank][t] on every rank: through the multicast address when
// mc_pairs != 0, else to each peer over P2P.
extern "C" __global__ void __launch_bounds__(512) fb_argmax_shard(
    const bf16* __restrict__ logits, long long ld, int T, int V, int vocab_offset, unsigned long long mc_pairs,
    unsigned long long base, unsigned long long stride, unsigned long long pairs_off, int rank, int world) {
  pdl_entry();
  const int t = blockIdx.x;
  if (t >= T) return;
  const bf16* row = logits + static_cast<size_t>(t) * ld;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
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
  if (threadIdx.x != 0) return;
  for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w)
    if (sb[w] > best || (sb[w] == best && si[w] < bi)) {
      best = sb[w];
      bi = si[w];
    }
  const uint32_t vbits = __float_as_uint(best);
  const uint32_t gidx = static_cast<uint32_t>(bi + vocab_offset);
  const uint64_t off = pairs_off + (static_cast<uint64_t>(rank) * T + t) * 8;
  if (mc_pairs) {
    asm volatile("multimem.st.relaxed.sys.global.b32 [%0], %1;" ::"l"(mc_pairs + off), "r"(vbits) : "memory");
    asm volatile("multimem.st.relaxed.sys.global.b32 [%0], %1;" ::"l"(mc_pairs + off + 4), "r"(gidx) : "memory");
  } else {
    for (int r = 0; r < world; ++r) {
      uint32_t* p = reinterpret_cast<uint32_t*>(base + r * stride + off);
      p[0] = vbits;
      p[1] = gidx;
    }
  }
}

extern "C" __global__ void fb_argmax_combine(const uint32_t* __restrict__ pairs, int T, int W, int* __restrict__ out) {
  pdl_entry();
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= T) return;
  float best = -INFINITY;
  uint32_t bi = 0x7fffffffu;
  for (int r = 0; r < W; ++r) {
    const uint32_t* p = pairs + (static_cast<size_t>(r) * T + t) * 2;
    const float v = __uint_as_float(__ldcv(p));
    const uint32_t i = __ldcv(p + 1);
    if (v > best || (v == best && i < bi)) {
      best = v;
      bi = i;
    }
  }
  out[t] = static_cast<int>(bi);
}

// Copies a local buffer to the same offset of every rank (P2P), for builds
// without multicast: the unfused fallback of the slot exchange.
extern "C" __global__ void fb_sym_broadcast(const uint4* __restrict__ src, unsigned long long base,
                                            unsigned long long stride, unsigned long long offset, long long nbytes,
                                            int world) {
  pdl_entry();
  const long long nv = nbytes / 16;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < nv;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const uint4 v = src[i];
    for (int r = 0; r < world; ++r) reinterpret_cast<uint4*>(base + r * stride + offset)[i] = v;
  }
}
