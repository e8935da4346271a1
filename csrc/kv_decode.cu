// Serving kernels: K15 paged KV-cache append (bf16 / fp8-e4m3 / int8 with a
// scale per (token, kv head)), K13 paged decode attention (split-KV with a
// combine pass, GQA query heads packed per CTA) and K19 sampling (greedy
// argmax, Gumbel-max temperature sampling).
//
// Cache layout per layer: K and V pages [num_blocks, block_size, Hkv, Dh] of
// the cache dtype, scales [num_blocks, block_size, Hkv] fp32 (quantized
// caches only).  A token's slot is block_id * block_size + offset; per
// sequence a block table maps logical block i to a physical block id, so
// sequences sharing a prefix can point at the same physical blocks.
//
// Replaces the reference's KVCache / PagedKVCache (include/nn/kv_cache.hpp:
// 12-219, a single global page table of fp32 copies), its KVCacheQuantizer
// (include/nn/quantization_production.hpp:293-316, truncating fake-quant) and
// the unreachable decode path of TransformerBlock::forward
// (src/nn/transformer_blocks.cpp:425-483, whose running softmax is wrong).
#include "common.cuh"
#include "host_util.h"
#include "lk_api.h"

namespace lk {

template <int KV>  // 0 bf16, 1 fp8 e4m3, 2 int8
struct KvT;
template <>
struct KvT<0> {
  using T = __nv_bfloat16;
  static constexpr float QMAX = 1.f;
};
template <>
struct KvT<1> {
  using T = __nv_fp8_e4m3;
  static constexpr float QMAX = 448.f;
};
template <>
struct KvT<2> {
  using T = int8_t;
  static constexpr float QMAX = 127.f;
};

template <int KV>
__device__ __forceinline__ typename KvT<KV>::T kv_encode(float x, float inv_scale) {
  if constexpr (KV == 0) {
    return __float2bfloat16(x);
  } else if constexpr (KV == 1) {
    return __nv_fp8_e4m3(x * inv_scale);  // saturating round-to-nearest-even
  } else {
    float q = rintf(x * inv_scale);
    q = fminf(fmaxf(q, -127.f), 127.f);
    return (int8_t)q;
  }
}

template <int KV>
__device__ __forceinline__ float kv_decode(typename KvT<KV>::T v) {
  if constexpr (KV == 0) return __bfloat162float(v);
  else if constexpr (KV == 1) return float(v);
  else return (float)v;
}

// One warp per (token, kv head, K|V): amax over Dh, scale, encode, store.
template <int KV>
__global__ void kv_append_kernel(const __nv_bfloat16* __restrict__ qkv, int64_t ld, int T, int Hq,
                                 int Hkv, int Dh, const int* __restrict__ slots,
                                 typename KvT<KV>::T* __restrict__ kc, typename KvT<KV>::T* __restrict__ vc,
                                 float* __restrict__ ks, float* __restrict__ vs, int num_slots,
                                 int* status) {
  const int64_t w = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= (int64_t)T * Hkv * 2) return;
  const int which = (int)(w & 1);  // 0 = K, 1 = V
  const int h = (int)((w >> 1) % Hkv);
  const int t = (int)((w >> 1) / Hkv);
  const int slot = slots[t];
  if (slot < 0) return;
  if (slot >= num_slots) {
    if (lane == 0 && status) atomicCAS(status, 0, LK_ERR_BAD_INDEX);
    return;
  }
  const __nv_bfloat16* src = qkv + (int64_t)t * ld + (Hq + which * Hkv + h) * Dh;
  float x[4];
  float amax = 0.f;
  const int per = Dh / 32;  // 2 or 4
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    x[i] = i < per ? __bfloat162float(src[lane * per + i]) : 0.f;
    amax = fmaxf(amax, fabsf(x[i]));
  }
  amax = warp_max(amax);
  const float scale = (KV == 0 || amax == 0.f) ? 1.f : amax / KvT<KV>::QMAX;
  const float inv = 1.f / scale;
  typename KvT<KV>::T* dst = (which ? vc : kc) + ((int64_t)slot * Hkv + h) * Dh;
#pragma unroll
  for (int i = 0; i < 4; ++i)
    if (i < per) dst[lane * per + i] = kv_encode<KV>(x[i], inv);
  if (KV != 0 && lane == 0) (which ? vs : ks)[(int64_t)slot * Hkv + h] = scale;
}

// Unpack N consecutive cache elements (N = 2, 4, 8, 16, 32; 16-byte aligned
// for N * sizeof >= 16) at p into floats (scale not applied).
template <int KV, int N>
__device__ __forceinline__ void kv_load(const typename KvT<KV>::T* p, float (&x)[N]) {
  constexpr int BYTES = N * (KV == 0 ? 2 : 1);
  uint32_t w[BYTES / 4 > 0 ? BYTES / 4 : 1];
  if constexpr (BYTES >= 16) {
#pragma unroll
    for (int i = 0; i < BYTES / 16; ++i) {
      const uint4 v = reinterpret_cast<const uint4*>(p)[i];
      w[4 * i] = v.x;
      w[4 * i + 1] = v.y;
      w[4 * i + 2] = v.z;
      w[4 * i + 3] = v.w;
    }
  } else if constexpr (BYTES == 8) {
    const uint2 v = *reinterpret_cast<const uint2*>(p);
    w[0] = v.x;
    w[1] = v.y;
  } else if constexpr (BYTES == 4) {
    w[0] = *reinterpret_cast<const uint32_t*>(p);
  } else {
    w[0] = *reinterpret_cast<const uint16_t*>(p);
  }
#pragma unroll
  for (int i = 0; i < N; ++i) {
    if constexpr (KV == 0) {
      const uint32_t h = (w[i / 2] >> (16 * (i & 1))) & 0xFFFFu;
      x[i] = __uint_as_float(h << 16);
    } else if constexpr (KV == 1) {
      const __nv_fp8_storage_t b = (__nv_fp8_storage_t)((w[i / 4] >> (8 * (i & 3))) & 0xFFu);
      x[i] = __half2float(__half(__nv_cvt_fp8_to_halfraw(b, __NV_E4M3)));
    } else {
      x[i] = (float)(int8_t)((w[i / 4] >> (8 * (i & 3))) & 0xFFu);
    }
  }
}

// Decode attention, split-KV (flash-decoding).  grid (num_splits, Hkv,
// num_seqs), 128 threads; a CTA handles the tokens [t0, t1) of one (sequence,
// kv head) for its G query heads.
//  phase 1  scores into shared memory: 8 lanes per token, each loading its
//           DH / 8 contiguous cache elements with 16-byte loads (a warp reads 4
//           whole K rows per step, four steps in flight) against its slice of
//           the G query rows, held in registers; 8-lane shuffle reduction;
//  phase 2  per-head max and sum over the split (block reductions);
//  phase 3  P V: 8 lanes per token (32 for G = 8) with 16-byte loads, four
//           tokens per warp step and four steps in flight; token groups and
//           then the four warps' partial outputs are added.
// Writes unnormalised partial outputs plus (max, sum) per (split, head) when
// num_splits > 1, else the final output.  A block id outside [0, num_blocks)
// (bounds-checked builds) is reported in *status and its tokens are skipped.
template <int KV, int DH, int G>
__global__ void __launch_bounds__(128) decode_attn_kernel(
    const __nv_bfloat16* __restrict__ q, int64_t ldq, const typename KvT<KV>::T* __restrict__ kc,
    const typename KvT<KV>::T* __restrict__ vc, const float* __restrict__ ks, const float* __restrict__ vs,
    const int* __restrict__ block_tables, int max_blocks, const int* __restrict__ ctx_lens,
    int block_size, int Hkv, float sl2, int split_len, __nv_bfloat16* __restrict__ out, int64_t ldo,
    float* __restrict__ part_o, float* __restrict__ part_ml, int num_splits, int num_blocks, int* status) {
  constexpr int LPT = 8;               // lanes per token in phase 1
  constexpr int DPL = DH / LPT;        // dims per lane in phase 1
  constexpr int TPI = 32 / LPT;        // tokens per warp step in phase 1
  extern __shared__ float sm[];
  float* sp = sm;  // [G][split_len] scores -> probabilities; reused for the phase-3 reduction
  __shared__ float red[G][4];
  const int split = blockIdx.x, kvh = blockIdx.y, seq = blockIdx.z;
  const int ctx = ctx_lens[seq];
  const int t0 = split * split_len;
  const int t1 = min(ctx, t0 + split_len);
  const int n = max(0, t1 - t0);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int* bt = block_tables + (int64_t)seq * max_blocks;
  auto slot_of = [&](int t, bool& ok) -> int64_t {
    const int blk = bt[t / block_size];
    ok = LK_BOUNDS(blk >= 0 && blk < num_blocks, status, LK_ERR_BAD_INDEX);
    return (int64_t)blk * block_size + (t % block_size);
  };
  // ---------------------------------------------------------------- phase 1
  {
    const int grp = lane / LPT, sub = lane % LPT;
    uint32_t qr[G][DPL / 2];  // this lane's dims of every query head, bf16 pairs
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const uint4* qp = reinterpret_cast<const uint4*>(q + (int64_t)seq * ldq + (kvh * G + g) * DH + sub * DPL);
#pragma unroll
      for (int i = 0; i < DPL / 8; ++i) {
        const uint4 v = qp[i];
        qr[g][4 * i] = v.x;
        qr[g][4 * i + 1] = v.y;
        qr[g][4 * i + 2] = v.z;
        qr[g][4 * i + 3] = v.w;
      }
    }
#pragma unroll(G <= 4 ? 4 : 2)
    for (int base = warp * TPI; base < n; base += 4 * TPI) {
      const int tt = base + grp;
      float sc[G];
#pragma unroll
      for (int g = 0; g < G; ++g) sc[g] = 0.f;
      bool ok = tt < n;
      if (ok) {
        const int64_t slot = slot_of(t0 + tt, ok);
        if (ok) {
          float x[DPL];
          kv_load<KV, DPL>(kc + (slot * Hkv + kvh) * DH + sub * DPL, x);
          const float kscale = (KV == 0 ? 1.f : ks[slot * Hkv + kvh]) * sl2;
#pragma unroll
          for (int g = 0; g < G; ++g) {
            float a = 0.f;
#pragma unroll
            for (int i = 0; i < DPL / 2; ++i) {
              const float2 qf = unpack_bf16x2(qr[g][i]);
              a = fmaf(qf.x, x[2 * i], fmaf(qf.y, x[2 * i + 1], a));
            }
            sc[g] = a * kscale;
          }
        }
      }
#pragma unroll
      for (int g = 0; g < G; ++g)
#pragma unroll
        for (int o = LPT / 2; o > 0; o >>= 1) sc[g] += __shfl_xor_sync(0xffffffffu, sc[g], o);
      if (tt < n && sub == 0)
#pragma unroll
        for (int g = 0; g < G; ++g) sp[g * split_len + tt] = ok ? sc[g] : -INFINITY;
    }
  }
  __syncthreads();
  // ---------------------------------------------------------------- phase 2
  float mx[G], sum[G];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float m = -INFINITY;
    for (int tt = tid; tt < n; tt += 128) m = fmaxf(m, sp[g * split_len + tt]);
    m = warp_max(m);
    if (lane == 0) red[g][warp] = m;
  }
  __syncthreads();
#pragma unroll
  for (int g = 0; g < G; ++g) mx[g] = fmaxf(fmaxf(red[g][0], red[g][1]), fmaxf(red[g][2], red[g][3]));
  __syncthreads();
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float sacc = 0.f;
    for (int tt = tid; tt < n; tt += 128) {
      const float p = mx[g] == -INFINITY ? 0.f : fast_exp2(sp[g * split_len + tt] - mx[g]);
      sp[g * split_len + tt] = p;
      sacc += p;
    }
    sacc = warp_sum(sacc);
    if (lane == 0) red[g][warp] = sacc;
  }
  __syncthreads();
#pragma unroll
  for (int g = 0; g < G; ++g) sum[g] = red[g][0] + red[g][1] + red[g][2] + red[g][3];
  // ---------------------------------------------------------------- phase 3
  // LP3 lanes per token (16-byte loads for G <= 4), TP3 tokens per warp step;
  // the token groups of a warp are added with shuffles at the end
  constexpr int LP3 = G <= 4 ? 8 : 32;
  constexpr int D3 = DH / LP3;
  constexpr int TP3 = 32 / LP3;
  const int g3 = lane / LP3, s3 = lane % LP3;
  float acc[G][D3];
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int j = 0; j < D3; ++j) acc[g][j] = 0.f;
#pragma unroll 4
  for (int base = warp * TP3; base < n; base += 4 * TP3) {
    const int tt = base + g3;
    if (tt < n) {
      bool ok;
      const int64_t slot = slot_of(t0 + tt, ok);
      if (ok) {
        float v[D3];
        kv_load<KV, D3>(vc + (slot * Hkv + kvh) * DH + s3 * D3, v);
        const float vscale = KV == 0 ? 1.f : vs[slot * Hkv + kvh];
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float p = sp[g * split_len + tt] * vscale;
#pragma unroll
          for (int j = 0; j < D3; ++j) acc[g][j] = fmaf(p, v[j], acc[g][j]);
        }
      }
    }
  }
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int j = 0; j < D3; ++j)
#pragma unroll
      for (int o = LP3; o < 32; o <<= 1) acc[g][j] += __shfl_xor_sync(0xffffffffu, acc[g][j], o);
  __syncthreads();  // sp is free: it holds the four warps' partial outputs now
  float* po = sm;   // [4][G][DH]
  if (g3 == 0)
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
      for (int j = 0; j < D3; ++j) po[(warp * G + g) * DH + s3 * D3 + j] = acc[g][j];
  __syncthreads();
  for (int i = tid; i < G * DH; i += 128) {
    const int g = i / DH, d = i % DH;
    const float o = po[i] + po[G * DH + i] + po[2 * G * DH + i] + po[3 * G * DH + i];
    const int h = kvh * G + g;
    if (num_splits == 1) {
      const float inv = sum[g] > 0.f ? 1.f / sum[g] : 0.f;
      out[(int64_t)seq * ldo + h * DH + d] = __float2bfloat16(o * inv);
    } else {
      part_o[(((int64_t)seq * (Hkv * G) + h) * num_splits + split) * DH + d] = o;
    }
  }
  if (num_splits > 1 && tid < G) {
    const int h = kvh * G + tid;
    float* ml = part_ml + (((int64_t)seq * (Hkv * G) + h) * num_splits + split) * 2;
    ml[0] = mx[tid];
    ml[1] = sum[tid];
  }
}

// Combine split partials: one warp per (seq, head).
template <int DH>
__global__ void decode_combine_kernel(const float* __restrict__ part_o, const float* __restrict__ part_ml,
                                      int num_seqs, int Hq, int num_splits, const int* __restrict__ ctx_lens,
                                      int split_len, __nv_bfloat16* __restrict__ out, int64_t ldo) {
  const int64_t w = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= (int64_t)num_seqs * Hq) return;
  const int seq = (int)(w / Hq), h = (int)(w % Hq);
  const int used = min(num_splits, (ctx_lens[seq] + split_len - 1) / split_len);
  const float* ml = part_ml + w * num_splits * 2;
  float M = -INFINITY;
  for (int s = 0; s < used; ++s) M = fmaxf(M, ml[2 * s]);
  float L = 0.f;
  float acc[DH / 32];
#pragma unroll
  for (int i = 0; i < DH / 32; ++i) acc[i] = 0.f;
  for (int s = 0; s < used; ++s) {
    const float m = ml[2 * s];
    const float f = m == -INFINITY ? 0.f : fast_exp2(m - M);
    L += ml[2 * s + 1] * f;
    const float* po = part_o + (w * num_splits + s) * DH;
#pragma unroll
    for (int i = 0; i < DH / 32; ++i) acc[i] += po[lane + 32 * i] * f;
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
#pragma unroll
  for (int i = 0; i < DH / 32; ++i)
    out[(int64_t)seq * ldo + h * DH + lane + 32 * i] = __float2bfloat16(acc[i] * inv);
}

// ------------------------------------------------ decode attention, paged TMA form
// Same contract as decode_attn_kernel (grid (num_splits, Hkv, num_seqs), same
// partial layout for the combine pass), built around an asynchronous page ring:
//   warp 4      producer: per KV page of the split, one 3-D TMA box for the
//               page's K rows of this KV head, one for its V rows, and bulk
//               copies of the page's K / V scales, into a ring of NS stages on
//               one mbarrier each; the block table is read 32 entries at a time;
//   warps 0-3   consumers, one pass with an online softmax per warp: LPT lanes
//               per token (16-byte shared-memory loads of the cached row), the
//               query slice in fp32 registers, packed f32x2 FMAs for q.k and
//               p.v, the running max rescaling the warp's accumulators only
//               when it grows; the four warps' (max, sum, output) are merged at
//               the end through shared memory.
// Pages are fetched whole; tokens outside [t0, t1) or past the context are
// masked.  A block id outside [0, num_blocks) (bounds-checked builds) is
// reported in *status and its page is skipped (no copy is issued).
constexpr int DEC_CONSUMERS = 4;
constexpr int DEC_THREADS = 32 * (DEC_CONSUMERS + 1);

struct DecLayout {
  int sk, ss, stage, ns, merge_off, bar_off, smem;
};

__host__ __device__ inline int dec_align128(int x) { return (x + 127) & ~127; }

__host__ __device__ inline DecLayout dec_layout(int bs, int DH, int esize, int Hkv, int G, bool scaled) {
  DecLayout L;
  L.sk = dec_align128(bs * DH * esize);
  L.ss = scaled ? dec_align128(bs * Hkv * 4) : 0;
  L.stage = 2 * L.sk + 2 * L.ss;
  int ns = (40 * 1024) / L.stage;
  L.ns = ns < 2 ? 2 : (ns > 12 ? 12 : ns);
  L.merge_off = L.ns * L.stage;
  const int merge = DEC_CONSUMERS * G * DH * 4 + 2 * DEC_CONSUMERS * G * 4;
  L.bar_off = dec_align128(L.merge_off + merge);
  L.smem = L.bar_off + 2 * L.ns * 8 + 4 * L.ns + 16 + 128;
  return L;
}

__device__ __forceinline__ void ffma2(float& a0, float& a1, float x0, float x1, float y0, float y1) {
  // (a0, a1) += (x0, x1) * (y0, y1) as one packed f32x2 FMA
  uint64_t a, x, y;
  asm("mov.b64 %0, {%1, %2};" : "=l"(a) : "f"(a0), "f"(a1));
  asm("mov.b64 %0, {%1, %2};" : "=l"(x) : "f"(x0), "f"(x1));
  asm("mov.b64 %0, {%1, %2};" : "=l"(y) : "f"(y0), "f"(y1));
  asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(a) : "l"(x), "l"(y));
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a0), "=f"(a1) : "l"(a));
}

// N cached values at shared address p -> floats (scale not applied)
template <int KV, int N>
__device__ __forceinline__ void kv_load_smem(const uint8_t* p, float (&x)[N]) {
  constexpr int BYTES = N * (KV == 0 ? 2 : 1);
  static_assert(BYTES % 2 == 0, "kv_load_smem: 2-byte multiples");
  uint32_t w[BYTES >= 4 ? BYTES / 4 : 1];
  if constexpr (BYTES >= 16) {
#pragma unroll
    for (int i = 0; i < BYTES / 16; ++i) {
      const uint4 v = reinterpret_cast<const uint4*>(p)[i];
      w[4 * i] = v.x, w[4 * i + 1] = v.y, w[4 * i + 2] = v.z, w[4 * i + 3] = v.w;
    }
  } else if constexpr (BYTES == 8) {
    const uint2 v = *reinterpret_cast<const uint2*>(p);
    w[0] = v.x, w[1] = v.y;
  } else if constexpr (BYTES == 4) {
    w[0] = *reinterpret_cast<const uint32_t*>(p);
  } else {
    w[0] = *reinterpret_cast<const uint16_t*>(p);
  }
#pragma unroll
  for (int i = 0; i < N; i += 2) {
    if constexpr (KV == 0) {
      const uint32_t u = w[i / 2];
      x[i] = __uint_as_float(u << 16);
      x[i + 1] = __uint_as_float(u & 0xFFFF0000u);
    } else if constexpr (KV == 1) {
      // two e4m3 codes -> f16x2 (exact) -> two floats
      const uint16_t pair = (uint16_t)(w[i / 4] >> (8 * (i & 3)));
      uint32_t h2;
      asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h2) : "h"(pair));
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h2));
      x[i] = f.x;
      x[i + 1] = f.y;
    } else {
      x[i] = (float)(int8_t)((w[i / 4] >> (8 * (i & 3))) & 0xFFu);
      x[i + 1] = (float)(int8_t)((w[i / 4] >> (8 * (i & 3) + 8)) & 0xFFu);
    }
  }
}

template <int KV, int DH, int G>
__global__ void __launch_bounds__(DEC_THREADS, 4) decode_attn_tma_kernel(
    const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
    const __nv_bfloat16* __restrict__ q, int64_t ldq, const float* __restrict__ ks, const float* __restrict__ vs,
    const int* __restrict__ block_tables, int max_blocks, const int* __restrict__ ctx_lens, int block_size,
    int Hkv, float sl2, int split_len, __nv_bfloat16* __restrict__ out, int64_t ldo, float* __restrict__ part_o,
    float* __restrict__ part_ml, int num_splits, int num_blocks, int* status) {
  constexpr int ES = KV == 0 ? 2 : 1;
  // lanes per token: the query slice and the accumulators stay at 2 * G * DH / LPT
  // registers per lane, so four CTAs fit per SM
  constexpr int LPT = G <= 2 ? 8 : (G == 4 ? 16 : 32);
  constexpr int DPL = DH / LPT;         // cached values per lane
  constexpr int TPW = 32 / LPT;         // tokens per warp step
  constexpr int TPS = TPW * DEC_CONSUMERS;
  extern __shared__ uint8_t dsm_raw[];
  uint8_t* dsm = dsm_raw + ((128 - (smem_u32(dsm_raw) & 127)) & 127);
  const int bs = block_size;
  const DecLayout L = dec_layout(bs, DH, ES, Hkv, G, KV != 0);
  const uint32_t sbase = smem_u32(dsm);
  const uint32_t full0 = sbase + L.bar_off, empty0 = full0 + 8 * L.ns;
  volatile int* stage_ok = reinterpret_cast<volatile int*>(dsm + L.bar_off + 16 * L.ns);
  volatile int* abort_flag = stage_ok + L.ns;
  const int split = blockIdx.x, kvh = blockIdx.y, seq = blockIdx.z;
  const int ctx = ctx_lens[seq];
  const int t0 = split * split_len;
  const int t1 = min(ctx, t0 + split_len);
  const int pg0 = t0 / bs;
  const int npg = t1 > t0 ? (t1 + bs - 1) / bs - pg0 : 0;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  if (tid == 0) {
    for (int i = 0; i < L.ns; ++i) {
      mbar_init(full0 + 8 * i, 1);
      mbar_init(empty0 + 8 * i, DEC_CONSUMERS);
    }
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  __syncthreads();

  if (warp == DEC_CONSUMERS) {
    // ------------------------------------------------------------ producer
    const int* bt = block_tables + (int64_t)seq * max_blocks;
    const uint32_t tx = 2u * bs * DH * ES + (KV != 0 ? 2u * bs * Hkv * 4 : 0u);
    uint32_t pending = 0, par = 0;
    int blk_lane = 0;
    for (int i = 0; i < npg; ++i) {
      if ((i & 31) == 0) blk_lane = i + lane < npg ? bt[pg0 + i + lane] : 0;
      const int blk = __shfl_sync(0xffffffffu, blk_lane, i & 31);
      const int s = i % L.ns;
      const uint32_t ph = (uint32_t)(i / L.ns) & 1;
      int ok = 1;
      if (lane == 0) {
        ok = bounded_wait(empty0 + 8 * s, ph ^ 1, status, LK_ERR_TIMEOUT_EMPTY, abort_flag);
        if (ok) {
          const bool valid = LK_BOUNDS(blk >= 0 && blk < num_blocks, status, LK_ERR_BAD_INDEX);
          stage_ok[s] = valid;
          if (valid) {
            const uint32_t st = sbase + s * L.stage;
            mbar_expect_tx(full0 + 8 * s, tx);
            tma_load_3d(st, &tmK, full0 + 8 * s, 0, kvh, blk * bs);
            tma_load_3d(st + L.sk, &tmV, full0 + 8 * s, 0, kvh, blk * bs);
            if constexpr (KV != 0) {
              bulk_load(st + 2 * L.sk, ks + (int64_t)blk * bs * Hkv, bs * Hkv * 4, full0 + 8 * s);
              bulk_load(st + 2 * L.sk + L.ss, vs + (int64_t)blk * bs * Hkv, bs * Hkv * 4, full0 + 8 * s);
            }
            pending |= 1u << s;
            par = (par & ~(1u << s)) | (ph << s);
          } else {
            mbar_arrive(full0 + 8 * s);
          }
        }
      }
      if (!__shfl_sync(0xffffffffu, ok, 0)) {
        if (lane == 0)
          for (int j = 0; j < L.ns; ++j)
            if (pending & (1u << j))
              bounded_wait(full0 + 8 * j, (par >> j) & 1, status, LK_ERR_TIMEOUT_DRAIN, nullptr);
        break;
      }
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  const int grp = lane / LPT, sub = lane % LPT;
  float qf[G][DPL];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const uint32_t* qp = reinterpret_cast<const uint32_t*>(q + (int64_t)seq * ldq + (kvh * G + g) * DH + sub * DPL);
#pragma unroll
    for (int i = 0; i < DPL / 2; ++i) {
      const float2 f = unpack_bf16x2(qp[i]);
      qf[g][2 * i] = f.x;
      qf[g][2 * i + 1] = f.y;
    }
  }
  float m[G], l[G], acc[G][DPL];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int d = 0; d < DPL; ++d) acc[g][d] = 0.f;
  }
  for (int i = 0; i < npg; ++i) {
    const int s = i % L.ns;
    const bool ok = bounded_wait(full0 + 8 * s, (uint32_t)(i / L.ns) & 1, status, LK_ERR_TIMEOUT_FULL, abort_flag);
    if (!__all_sync(0xffffffffu, ok)) break;
    const bool page_ok = stage_ok[s] != 0;
    const uint8_t* st = dsm + s * L.stage;
    const int tp = (pg0 + i) * bs;
    for (int j0 = 0; j0 < bs; j0 += TPS) {
      const int j = j0 + warp * TPW + grp;
      const int tt = tp + j;
      const bool tok = page_ok && j < bs && tt >= t0 && tt < t1;
      float sc[G];
#pragma unroll
      for (int g = 0; g < G; ++g) sc[g] = 0.f;
      if (tok) {
        float x[DPL];
        kv_load_smem<KV, DPL>(st + (j * DH + sub * DPL) * ES, x);
        const float kscale = (KV == 0 ? 1.f : reinterpret_cast<const float*>(st + 2 * L.sk)[j * Hkv + kvh]) * sl2;
#pragma unroll
        for (int g = 0; g < G; ++g) {
          float a0 = 0.f, a1 = 0.f;
#pragma unroll
          for (int d = 0; d < DPL; d += 2) ffma2(a0, a1, qf[g][d], qf[g][d + 1], x[d], x[d + 1]);
          sc[g] = (a0 + a1) * kscale;
        }
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
#pragma unroll
        for (int o = LPT / 2; o > 0; o >>= 1) sc[g] += __shfl_xor_sync(0xffffffffu, sc[g], o);
      }
      float p[G];
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float tmax = tok ? sc[g] : -INFINITY;
#pragma unroll
        for (int o = LPT; o < 32; o <<= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, o));
        if (tmax > m[g]) {  // warp-uniform: the running max grows
          const float alpha = m[g] == -INFINITY ? 0.f : fast_exp2(m[g] - tmax);
          l[g] *= alpha;
#pragma unroll
          for (int d = 0; d < DPL; ++d) acc[g][d] *= alpha;
          m[g] = tmax;
        }
        p[g] = tok ? fast_exp2(sc[g] - m[g]) : 0.f;
        l[g] += p[g];
      }
      if (tok) {
        float v[DPL];
        kv_load_smem<KV, DPL>(st + L.sk + (j * DH + sub * DPL) * ES, v);
        const float vscale = KV == 0 ? 1.f : reinterpret_cast<const float*>(st + 2 * L.sk + L.ss)[j * Hkv + kvh];
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float pv = p[g] * vscale;
#pragma unroll
          for (int d = 0; d < DPL; d += 2) ffma2(acc[g][d], acc[g][d + 1], pv, pv, v[d], v[d + 1]);
        }
      }
    }
    fence_proxy_async_smem();  // generic reads of the stage before its async-proxy (TMA) refill
    __syncwarp();
    if (lane == 0) mbar_arrive(empty0 + 8 * s);
  }
  // token groups of the warp -> one (sum, output) per warp
#pragma unroll
  for (int g = 0; g < G; ++g) {
#pragma unroll
    for (int o = LPT; o < 32; o <<= 1) {
      l[g] += __shfl_xor_sync(0xffffffffu, l[g], o);
#pragma unroll
      for (int d = 0; d < DPL; ++d) acc[g][d] += __shfl_xor_sync(0xffffffffu, acc[g][d], o);
    }
  }
  float* po = reinterpret_cast<float*>(dsm + L.merge_off);  // [4][G][DH]
  float* pm = po + DEC_CONSUMERS * G * DH;                   // [4][G]
  float* pl = pm + DEC_CONSUMERS * G;                        // [4][G]
  if (grp == 0)
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
      for (int d = 0; d < DPL; ++d) po[(warp * G + g) * DH + sub * DPL + d] = acc[g][d];
  if (lane == 0)
#pragma unroll
    for (int g = 0; g < G; ++g) {
      pm[warp * G + g] = m[g];
      pl[warp * G + g] = l[g];
    }
  asm volatile("bar.sync 1, %0;" ::"n"(32 * DEC_CONSUMERS) : "memory");
  for (int idx = tid; idx < G * DH; idx += 32 * DEC_CONSUMERS) {
    const int g = idx / DH, d = idx % DH;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < DEC_CONSUMERS; ++w) M = fmaxf(M, pm[w * G + g]);
    float o = 0.f, S = 0.f;
#pragma unroll
    for (int w = 0; w < DEC_CONSUMERS; ++w) {
      const float mw = pm[w * G + g];
      const float f = mw == -INFINITY ? 0.f : fast_exp2(mw - M);
      o += po[(w * G + g) * DH + d] * f;
      S += pl[w * G + g] * f;
    }
    const int h = kvh * G + g;
    if (num_splits == 1) {
      out[(int64_t)seq * ldo + h * DH + d] = __float2bfloat16(S > 0.f ? o / S : 0.f);
    } else {
      part_o[(((int64_t)seq * (Hkv * G) + h) * num_splits + split) * DH + d] = o;
      if (d == 0) {
        float* ml = part_ml + (((int64_t)seq * (Hkv * G) + h) * num_splits + split) * 2;
        ml[0] = M;
        ml[1] = S;
      }
    }
  }
}

// Gather a sequence's cached K/V (token t at slot slots[t]) into contiguous
// bf16 rows [n, 2*Hkv*Dh]: keys in columns [0, Hkv*Dh), values after.
template <int KV>
__global__ void kv_gather_kernel(const typename KvT<KV>::T* __restrict__ kc, const typename KvT<KV>::T* __restrict__ vc,
                                 const float* __restrict__ ks, const float* __restrict__ vs,
                                 const int* __restrict__ slots, int n, int Hkv, int Dh,
                                 __nv_bfloat16* __restrict__ out, int64_t ldo, int num_slots, int* status) {
  const int64_t total = (int64_t)n * 2 * Hkv * Dh;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int d = (int)(idx % Dh);
    const int64_t r = idx / Dh;
    const int h = (int)(r % Hkv);
    const int which = (int)((r / Hkv) & 1);
    const int t = (int)(r / (2 * Hkv));
    const int64_t slot = slots[t];
    float v = 0.f;
    if (LK_BOUNDS(slot >= 0 && slot < num_slots, status, LK_ERR_BAD_INDEX)) {
      const int64_t src = (slot * Hkv + h) * Dh + d;
      v = kv_decode<KV>((which ? vc : kc)[src]);
      if (KV != 0) v *= (which ? vs : ks)[slot * Hkv + h];
    }
    out[(int64_t)t * ldo + (which * Hkv + h) * Dh + d] = __float2bfloat16(v);
  }
}

// ---------------------------------------------------------------- sampling
// Greedy: argmax per row (ties -> lowest index).  Temperature > 0: Gumbel-max
// with a counter-based hash of (seed, row, column), i.e. an exact sample from
// softmax(logits / temperature).
__device__ __forceinline__ uint32_t mix32(uint32_t x) {
  // 32-bit finaliser of a multiply-xorshift hash (public-domain "lowbias32")
  x ^= x >> 16;
  x *= 0x7feb352dU;
  x ^= x >> 15;
  x *= 0x846ca68bU;
  x ^= x >> 16;
  return x;
}

__global__ void sample_kernel(const __nv_bfloat16* __restrict__ logits, int64_t ld, int V,
                              const float* __restrict__ temperature, uint64_t seed,
                              int64_t* __restrict__ out_tok, float* __restrict__ out_val, int64_t v0) {
  const int row = blockIdx.x;
  const float temp = temperature ? temperature[row] : 0.f;
  const __nv_bfloat16* z = logits + (int64_t)row * ld;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int j = threadIdx.x; j < V; j += blockDim.x) {
    float v = __bfloat162float(z[j]);
    if (temp > 0.f) {
      const uint32_t h = mix32((uint32_t)seed ^ mix32((uint32_t)(seed >> 32) + row * 0x9e3779b9U) ^
                               mix32((uint32_t)(j + v0) * 0x85ebca6bU + 0x1234567U));
      const float u = ((h >> 8) + 0.5f) * (1.0f / 16777216.0f);  // (0, 1)
      v = v / temp - logf(-logf(u));
    }
    if (v > best || (v == best && j < bi)) {
      best = v;
      bi = j;
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
  __shared__ float sb[32];
  __shared__ int si[32];
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sb[w] = best;
    si[w] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int k = 1; k < (int)(blockDim.x >> 5); ++k)
      if (sb[k] > best || (sb[k] == best && si[k] < bi)) {
        best = sb[k];
        bi = si[k];
      }
    out_tok[row] = bi + v0;
    if (out_val) out_val[row] = best;
  }
}

// Nucleus (top-p) sampling, one block per row.  For rows with temperature T > 0
// and top_p p < 1 the nucleus is the smallest set of highest-scoring tokens whose
// softmax(z / T) mass reaches p: the block finds the threshold t with a
// bisection on the logit value (mass(t) = sum over z >= t of exp((z - max) / T),
// monotone in t) between max - 40 T (below which a token's weight is under
// e^-40) and max, 32 halvings, keeping mass(lo) >= p * total.  Bisection ends
// far inside one bf16 spacing, so the set {z >= t} is the exact nucleus.  The
// token is then the Gumbel-max over the nucleus with the same noise as
// sample_kernel, which is an exact draw from the renormalised nucleus
// distribution.  Rows with T <= 0 are greedy; rows with p >= 1 sample from
// the whole vocabulary, as sample_kernel does.  With row_seeds, row r's noise
// comes from row_seeds[r] alone (a request's draws then do not depend on which
// batch row it lands in).
__device__ __forceinline__ float block_reduce_topp(float v, bool is_max, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float w = __shfl_xor_sync(0xffffffffu, v, o);
    v = is_max ? fmaxf(v, w) : v + w;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();  // red[] may still be read by the previous reduction
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float r = is_max ? -INFINITY : 0.f;
  for (int k = 0; k < nw; ++k) r = is_max ? fmaxf(r, red[k]) : r + red[k];
  return r;
}

__global__ void sample_topp_kernel(const __nv_bfloat16* __restrict__ logits, int64_t ld, int V,
                                   const float* __restrict__ temperature, const float* __restrict__ top_p,
                                   uint64_t seed, const uint64_t* __restrict__ row_seeds,
                                   int64_t* __restrict__ out_tok) {
  __shared__ float red[32];
  const int row = blockIdx.x;
  const float temp = temperature ? temperature[row] : 0.f;
  const float p = top_p ? top_p[row] : 1.f;
  const __nv_bfloat16* z = logits + (int64_t)row * ld;
  float thr = -INFINITY;
  if (temp > 0.f && p < 1.f) {
    float m = -INFINITY;
    for (int j = threadIdx.x; j < V; j += blockDim.x) m = fmaxf(m, __bfloat162float(z[j]));
    m = block_reduce_topp(m, true, red);
    const float inv_t = 1.f / temp;
    float tot = 0.f;
    for (int j = threadIdx.x; j < V; j += blockDim.x) tot += __expf((__bfloat162float(z[j]) - m) * inv_t);
    tot = block_reduce_topp(tot, false, red);
    const float target = p * tot;
    float lo = m - 40.f * temp, hi = m;
#pragma unroll 1
    for (int it = 0; it < 32; ++it) {
      const float mid = 0.5f * (lo + hi);
      float mass = 0.f;
      for (int j = threadIdx.x; j < V; j += blockDim.x) {
        const float v = __bfloat162float(z[j]);
        if (v >= mid) mass += __expf((v - m) * inv_t);
      }
      mass = block_reduce_topp(mass, false, red);
      if (mass >= target) lo = mid;  // every thread holds the same sums, so the same branch
      else hi = mid;
    }
    thr = lo;
  }
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int j = threadIdx.x; j < V; j += blockDim.x) {
    float v = __bfloat162float(z[j]);
    if (v < thr) continue;
    if (temp > 0.f) {
      // without per-row seeds the noise is sample_kernel's, keyed by (seed, row);
      // a per-row seed (a request's own stream) replaces that key
      const uint32_t base = row_seeds
          ? mix32((uint32_t)row_seeds[row] ^ mix32((uint32_t)(row_seeds[row] >> 32)))
          : (uint32_t)seed ^ mix32((uint32_t)(seed >> 32) + row * 0x9e3779b9U);
      const uint32_t h = mix32(base ^ mix32((uint32_t)j * 0x85ebca6bU + 0x1234567U));
      const float u = ((h >> 8) + 0.5f) * (1.0f / 16777216.0f);  // (0, 1)
      v = v / temp - logf(-logf(u));
    }
    if (v > best || (v == best && j < bi)) {
      best = v;
      bi = j;
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
  __shared__ float sb[32];
  __shared__ int si[32];
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sb[w] = best;
    si[w] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int k = 1; k < (int)(blockDim.x >> 5); ++k)
      if (sb[k] > best || (sb[k] == best && si[k] < bi)) {
        best = sb[k];
        bi = si[k];
      }
    out_tok[row] = bi;
  }
}

// Paged TMA form (default); false when this launch cannot use it.
static bool decode_tma_ok(const LkDecodeDesc& d) {
  static const bool v1 = [] {
    const char* e = getenv("LK_DECODE_V1");
    return e && e[0] == '1';
  }();
  return !v1 && d.block_size % 4 == 0 && d.block_size <= 256 && d.num_blocks > 0;
}

template <int KV, int DH>
static int launch_decode_tma(const LkDecodeDesc& d, int G, int nsplit, cudaStream_t s) {
  constexpr int ES = KV == 0 ? 2 : 1;
  const DecLayout L = dec_layout(d.block_size, DH, ES, d.Hkv, G, KV != 0);
  const CUtensorMapDataType dt = KV == 0 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8;
  const int64_t slots = (int64_t)d.num_blocks * d.block_size;
  CUtensorMap tk, tv;
  if (!make_tmap_3d(&tk, d.k_cache, dt, ES, DH, d.Hkv, slots, (int64_t)DH * ES, (int64_t)d.Hkv * DH * ES, DH, 1,
                    d.block_size) ||
      !make_tmap_3d(&tv, d.v_cache, dt, ES, DH, d.Hkv, slots, (int64_t)DH * ES, (int64_t)d.Hkv * DH * ES, DH, 1,
                    d.block_size))
    return -1;
  dim3 grid(nsplit, d.Hkv, d.num_seqs);
  const float sl2 = d.scale * 1.4426950408889634f;
#define LK_DEC2(GG)                                                                                        \
  {                                                                                                        \
    auto k = decode_attn_tma_kernel<KV, DH, GG>;                                                           \
    if (L.smem > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, L.smem);  \
    k<<<grid, DEC_THREADS, L.smem, s>>>(tk, tv, (const __nv_bfloat16*)d.q, d.ldq, d.k_scale, d.v_scale,    \
                                        d.block_tables, d.max_blocks, d.ctx_lens, d.block_size, d.Hkv, sl2, \
                                        d.split_len, (__nv_bfloat16*)d.out, d.ldo, d.part_o, d.part_ml,    \
                                        nsplit, d.num_blocks, d.status);                                   \
    break;                                                                                                 \
  }
  switch (G) {
    case 1: LK_DEC2(1)
    case 2: LK_DEC2(2)
    case 4: LK_DEC2(4)
    case 8: LK_DEC2(8)
    default: return fail("decode_attention: GQA group must be 1, 2, 4 or 8");
  }
#undef LK_DEC2
  if (check_launch("decode_attn_tma")) return -1;
  if (nsplit > 1) {
    const int64_t warps = (int64_t)d.num_seqs * d.Hkv * G;
    decode_combine_kernel<DH><<<cdiv(warps * 32, 256), 256, 0, s>>>(
        d.part_o, d.part_ml, d.num_seqs, d.Hkv * G, nsplit, d.ctx_lens, d.split_len,
        (__nv_bfloat16*)d.out, d.ldo);
    return check_launch("decode_combine");
  }
  return 0;
}

template <int KV, int DH>
static int launch_decode_g(const LkDecodeDesc& d, int G, int nsplit, int smem, cudaStream_t s) {
  if (decode_tma_ok(d)) return launch_decode_tma<KV, DH>(d, G, nsplit, s);
  dim3 grid(nsplit, d.Hkv, d.num_seqs);
  const float sl2 = d.scale * 1.4426950408889634f;
  using T = typename KvT<KV>::T;
#define LK_DEC(GG)                                                                                   \
  {                                                                                                  \
    auto k = decode_attn_kernel<KV, DH, GG>;                                                         \
    if (smem > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem); \
    k<<<grid, 128, smem, s>>>((const __nv_bfloat16*)d.q, d.ldq, (const T*)d.k_cache, (const T*)d.v_cache, \
                              d.k_scale, d.v_scale, d.block_tables, d.max_blocks, d.ctx_lens,        \
                              d.block_size, d.Hkv, sl2, d.split_len, (__nv_bfloat16*)d.out, d.ldo,   \
                              d.part_o, d.part_ml, nsplit, d.num_blocks, d.status);                  \
    break;                                                                                           \
  }
  switch (G) {
    case 1: LK_DEC(1)
    case 2: LK_DEC(2)
    case 4: LK_DEC(4)
    case 8: LK_DEC(8)
    default: return fail("decode_attention: GQA group must be 1, 2, 4 or 8");
  }
#undef LK_DEC
  if (check_launch("decode_attn")) return -1;
  if (nsplit > 1) {
    const int64_t warps = (int64_t)d.num_seqs * d.Hkv * G;
    decode_combine_kernel<DH><<<cdiv(warps * 32, 256), 256, 0, s>>>(
        d.part_o, d.part_ml, d.num_seqs, d.Hkv * G, nsplit, d.ctx_lens, d.split_len,
        (__nv_bfloat16*)d.out, d.ldo);
    return check_launch("decode_combine");
  }
  return 0;
}

}  // namespace lk

using namespace lk;

extern "C" int lk_kv_append(const LkKvAppendDesc* d, cudaStream_t s) {
  LK_REQUIRE(d->Dh == 64 || d->Dh == 128, "kv_append: head_dim must be 64 or 128");
  const int64_t warps = (int64_t)d->T * d->Hkv * 2;
  if (warps == 0) return 0;
  const int grid = cdiv(warps * 32, 256);
  switch (d->kv_dtype) {
    case 0:
      kv_append_kernel<0><<<grid, 256, 0, s>>>((const __nv_bfloat16*)d->qkv, d->ld, d->T, d->Hq, d->Hkv, d->Dh,
                                               d->slots, (__nv_bfloat16*)d->k_cache, (__nv_bfloat16*)d->v_cache,
                                               nullptr, nullptr, d->num_slots, d->status);
      break;
    case 1:
      kv_append_kernel<1><<<grid, 256, 0, s>>>((const __nv_bfloat16*)d->qkv, d->ld, d->T, d->Hq, d->Hkv, d->Dh,
                                               d->slots, (__nv_fp8_e4m3*)d->k_cache, (__nv_fp8_e4m3*)d->v_cache,
                                               d->k_scale, d->v_scale, d->num_slots, d->status);
      break;
    case 2:
      kv_append_kernel<2><<<grid, 256, 0, s>>>((const __nv_bfloat16*)d->qkv, d->ld, d->T, d->Hq, d->Hkv, d->Dh,
                                               d->slots, (int8_t*)d->k_cache, (int8_t*)d->v_cache, d->k_scale,
                                               d->v_scale, d->num_slots, d->status);
      break;
    default:
      return fail("kv_append: kv_dtype must be 0 (bf16), 1 (fp8) or 2 (int8)");
  }
  return check_launch("kv_append");
}

extern "C" int lk_decode_attention(const LkDecodeDesc* d, cudaStream_t s) {
  LK_REQUIRE(d->Dh == 64 || d->Dh == 128, "decode_attention: head_dim must be 64 or 128");
  LK_REQUIRE(d->Hq % d->Hkv == 0, "decode_attention: Hq % Hkv");
  LK_REQUIRE(d->split_len > 0 && d->split_len <= 1024, "decode_attention: split_len in (0, 1024]");
  if (d->num_seqs == 0) return 0;
  const int G = d->Hq / d->Hkv;
  const int nsplit = d->num_splits;
  LK_REQUIRE(nsplit == 1 || (d->part_o && d->part_ml), "decode_attention: split partial buffers needed");
  // scores [G][split_len], later the four warps' partial outputs [4][G][Dh]
  const int smem = std::max(G * d->split_len, 4 * G * d->Dh) * (int)sizeof(float);
  if (d->kv_dtype == 0)
    return d->Dh == 64 ? launch_decode_g<0, 64>(*d, G, nsplit, smem, s) : launch_decode_g<0, 128>(*d, G, nsplit, smem, s);
  if (d->kv_dtype == 1)
    return d->Dh == 64 ? launch_decode_g<1, 64>(*d, G, nsplit, smem, s) : launch_decode_g<1, 128>(*d, G, nsplit, smem, s);
  if (d->kv_dtype == 2)
    return d->Dh == 64 ? launch_decode_g<2, 64>(*d, G, nsplit, smem, s) : launch_decode_g<2, 128>(*d, G, nsplit, smem, s);
  return fail("decode_attention: bad kv_dtype");
}

extern "C" int lk_kv_gather_checked(const void* k_cache, const void* v_cache, const float* k_scale,
                                    const float* v_scale, const int* slots, int n, int Hkv, int Dh, void* out,
                                    int64_t ldo, int kv_dtype, int num_slots, int* status, cudaStream_t s) {
  const int64_t work = (int64_t)n * 2 * Hkv * Dh;
  if (work == 0) return 0;
  const int grid = (int)std::min<int64_t>((work + 255) / 256, (int64_t)num_sms() * 8);
  if (kv_dtype == 0)
    kv_gather_kernel<0><<<grid, 256, 0, s>>>((const __nv_bfloat16*)k_cache, (const __nv_bfloat16*)v_cache, k_scale,
                                             v_scale, slots, n, Hkv, Dh, (__nv_bfloat16*)out, ldo, num_slots, status);
  else if (kv_dtype == 1)
    kv_gather_kernel<1><<<grid, 256, 0, s>>>((const __nv_fp8_e4m3*)k_cache, (const __nv_fp8_e4m3*)v_cache, k_scale,
                                             v_scale, slots, n, Hkv, Dh, (__nv_bfloat16*)out, ldo, num_slots, status);
  else
    kv_gather_kernel<2><<<grid, 256, 0, s>>>((const int8_t*)k_cache, (const int8_t*)v_cache, k_scale, v_scale,
                                             slots, n, Hkv, Dh, (__nv_bfloat16*)out, ldo, num_slots, status);
  return check_launch("kv_gather");
}

extern "C" int lk_kv_gather(const void* k_cache, const void* v_cache, const float* k_scale,
                            const float* v_scale, const int* slots, int n, int Hkv, int Dh, void* out,
                            int64_t ldo, int kv_dtype, cudaStream_t s) {
  return lk_kv_gather_checked(k_cache, v_cache, k_scale, v_scale, slots, n, Hkv, Dh, out, ldo, kv_dtype,
                              INT32_MAX, nullptr, s);
}

extern "C" int lk_sample(const void* logits, int64_t ld, int rows, int V, const float* temperature,
                         uint64_t seed, int64_t* out_tok, float* out_val, cudaStream_t s) {
  return lk_sample_vp(logits, ld, rows, V, 0, temperature, seed, out_tok, out_val, s);
}

extern "C" int lk_sample_topp(const void* logits, int64_t ld, int rows, int V, const float* temperature,
                              const float* top_p, uint64_t seed, const uint64_t* row_seeds, int64_t* out_tok,
                              cudaStream_t s) {
  LK_REQUIRE(V > 0, "sample_topp: empty vocabulary");
  if (rows == 0) return 0;
  sample_topp_kernel<<<rows, 512, 0, s>>>((const __nv_bfloat16*)logits, ld, V, temperature, top_p, seed, row_seeds,
                                          out_tok);
  return check_launch("sample_topp");
}

// Vocabulary-parallel form: the logits hold columns [v0, v0 + V) of the
// vocabulary; tokens come back as global ids and the Gumbel noise is drawn for
// the global id, so the best (value, id) over every rank's slice is exactly
// the single-GPU sample.
extern "C" int lk_sample_vp(const void* logits, int64_t ld, int rows, int V, int64_t v0,
                            const float* temperature, uint64_t seed, int64_t* out_tok, float* out_val,
                            cudaStream_t s) {
  if (rows == 0) return 0;
  sample_kernel<<<rows, 512, 0, s>>>((const __nv_bfloat16*)logits, ld, V, temperature, seed, out_tok, out_val,
                                     v0);
  return check_launch("sample");
}
