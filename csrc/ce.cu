// K9: softmax cross-entropy over vocabulary logits, loss + gradient in one
// kernel, the gradient written in place over the bf16 logits so no fp32 logits
// tensor is ever materialised.
//
//   loss_t  = (1-eps)(lse - z[t]) + eps(lse - mean_j z_j) + zl * lse^2
//   dz_j    = (p_j (1 + 2 zl lse) - (1-eps)[j == t] - eps/V) * scale
// with scale = (*scale_ptr) * scale_mul (the device-resident loss scale times
// 1/(tokens * accumulation steps)).  Rows whose target equals ignore_index
// contribute no loss and a zero gradient.
//
// Reference: the pipeline's inline CE+grad (include/nn/training_pipeline.hpp:74-98),
// FusedSoftmaxCrossEntropy (include/nn/optimizer_and_loss.hpp:85-102) and
// LabelSmoothing (include/nn/training_enhancements.hpp:167-192).
#include "common.cuh"
#include "host_util.h"
#include "lk_api.h"

namespace lk {

struct MS {
  float m, s;
};

__device__ __forceinline__ MS ms_combine(MS a, MS b) {
  const float m = fmaxf(a.m, b.m);
  if (m == -INFINITY) return {m, 0.f};
  return {m, a.s * __expf(a.m - m) + b.s * __expf(b.m - m)};
}

template <int THREADS>
__global__ void __launch_bounds__(THREADS) ce_kernel(__nv_bfloat16* __restrict__ logits, int64_t ld,
                                                     const int64_t* __restrict__ targets, int T, int V,
                                                     float* __restrict__ loss_acc, float* __restrict__ row_loss,
                                                     const float* __restrict__ scale_ptr, float scale_mul,
                                                     float smoothing, float zloss, int64_t ignore_index,
                                                     int write_grad) {
  __shared__ MS red_ms[THREADS / 32];
  __shared__ float red_sum[THREADS / 32];
  __shared__ float bcast[2];
  const int row = blockIdx.x;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  __nv_bfloat16* z = logits + (int64_t)row * ld;
  const int64_t tgt = targets[row];
  const bool ignored = (tgt == ignore_index) || tgt < 0 || tgt >= V;
  const int nvec = V / 8;

  MS acc{-INFINITY, 0.f};
  float zsum = 0.f;
  for (int i = threadIdx.x; i < nvec; i += THREADS) {
    const uint4 v = reinterpret_cast<const uint4*>(z)[i];
    const uint32_t vw[4] = {v.x, v.y, v.z, v.w};
    float f[8];
    float mx = -INFINITY;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 a = unpack_bf16x2(vw[e]);
      f[2 * e] = a.x;
      f[2 * e + 1] = a.y;
      mx = fmaxf(mx, fmaxf(a.x, a.y));
    }
    float s = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      s += __expf(f[e] - mx);
      zsum += f[e];
    }
    acc = ms_combine(acc, MS{mx, s});
  }
  // warp + block reduction of (max, sum) and of sum(z)
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    MS other{__shfl_xor_sync(0xffffffffu, acc.m, o), __shfl_xor_sync(0xffffffffu, acc.s, o)};
    acc = ms_combine(acc, other);
  }
  zsum = warp_sum(zsum);
  if (lane == 0) {
    red_ms[w] = acc;
    red_sum[w] = zsum;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    MS t = red_ms[0];
    float zs = red_sum[0];
    for (int k = 1; k < THREADS / 32; ++k) {
      t = ms_combine(t, red_ms[k]);
      zs += red_sum[k];
    }
    const float lse = t.m + logf(t.s);
    bcast[0] = lse;
    float loss = 0.f;
    if (!ignored) {
      const float zt = __bfloat162float(z[tgt]);
      loss = (1.f - smoothing) * (lse - zt) + smoothing * (lse - zs / (float)V) + zloss * lse * lse;
      atomicAdd(loss_acc, loss);
      atomicAdd(loss_acc + 1, 1.f);
    }
    if (row_loss) row_loss[row] = loss;
  }
  __syncthreads();
  if (!write_grad) return;
  const float lse = bcast[0];
  const float scale = ignored ? 0.f : (scale_ptr ? *scale_ptr : 1.f) * scale_mul;
  const float pmul = 1.f + 2.f * zloss * lse;
  const float off = smoothing / (float)V;
  for (int i = threadIdx.x; i < nvec; i += THREADS) {
    uint4 v = reinterpret_cast<const uint4*>(z)[i];
    uint32_t vw[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 a = unpack_bf16x2(vw[e]);
      const int j0 = i * 8 + 2 * e;
      float g0 = __expf(a.x - lse) * pmul - off;
      float g1 = __expf(a.y - lse) * pmul - off;
      if (j0 == tgt) g0 -= (1.f - smoothing);
      if (j0 + 1 == tgt) g1 -= (1.f - smoothing);
      vw[e] = pack_bf16x2(g0 * scale, g1 * scale);
    }
    reinterpret_cast<uint4*>(z)[i] = make_uint4(vw[0], vw[1], vw[2], vw[3]);
  }
}

// Vocabulary-parallel phase 1: partial statistics of the local columns.
template <int THREADS>
__global__ void __launch_bounds__(THREADS) ce_vp_stats_kernel(LkCeVpDesc d) {
  __shared__ MS red_ms[THREADS / 32];
  __shared__ float red_sum[THREADS / 32];
  const int row = blockIdx.x;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const __nv_bfloat16* z = reinterpret_cast<const __nv_bfloat16*>(d.ce.logits) + (int64_t)row * d.ce.ld;
  const int nvec = d.ce.V / 8;
  MS acc{-INFINITY, 0.f};
  float zsum = 0.f;
  for (int i = threadIdx.x; i < nvec; i += THREADS) {
    const uint4 v = reinterpret_cast<const uint4*>(z)[i];
    const uint32_t vw[4] = {v.x, v.y, v.z, v.w};
    float f[8];
    float mx = -INFINITY;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 a = unpack_bf16x2(vw[e]);
      f[2 * e] = a.x;
      f[2 * e + 1] = a.y;
      mx = fmaxf(mx, fmaxf(a.x, a.y));
    }
    float s = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      s += __expf(f[e] - mx);
      zsum += f[e];
    }
    acc = ms_combine(acc, MS{mx, s});
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    MS other{__shfl_xor_sync(0xffffffffu, acc.m, o), __shfl_xor_sync(0xffffffffu, acc.s, o)};
    acc = ms_combine(acc, other);
  }
  zsum = warp_sum(zsum);
  if (lane == 0) {
    red_ms[w] = acc;
    red_sum[w] = zsum;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    MS t = red_ms[0];
    float zs = red_sum[0];
    for (int k = 1; k < THREADS / 32; ++k) {
      t = ms_combine(t, red_ms[k]);
      zs += red_sum[k];
    }
    const int64_t tgt = d.ce.targets[row] - d.v0;
    const float zt = (tgt >= 0 && tgt < d.ce.V) ? __bfloat162float(z[tgt]) : 0.f;
    reinterpret_cast<float4*>(d.stats)[row] = make_float4(t.m, t.s, zs, zt);
  }
}

// Phase 2: combine every rank's statistics, loss, local gradient slice.
template <int THREADS>
__global__ void __launch_bounds__(THREADS) ce_vp_finish_kernel(LkCeVpDesc d) {
  __shared__ float bcast;
  const int row = blockIdx.x;
  __nv_bfloat16* z = reinterpret_cast<__nv_bfloat16*>(d.ce.logits) + (int64_t)row * d.ce.ld;
  const int64_t tg = d.ce.targets[row];
  const bool ignored = (tg == d.ce.ignore_index) || tg < 0 || tg >= d.V_total;
  if (threadIdx.x == 0) {
    MS t{-INFINITY, 0.f};
    float zs = 0.f, zt = 0.f;
    for (int p = 0; p < d.world; ++p) {  // fixed rank order: identical on every rank
      const float4 st = reinterpret_cast<const float4*>(d.peer_stats[p])[row];
      t = ms_combine(t, MS{st.x, st.y});
      zs += st.z;
      zt += st.w;
    }
    const float lse = t.m + logf(t.s);
    bcast = lse;
    float loss = 0.f;
    if (!ignored) {
      const float eps = d.ce.smoothing;
      loss = (1.f - eps) * (lse - zt) + eps * (lse - zs / (float)d.V_total) + d.ce.zloss * lse * lse;
      atomicAdd(d.ce.loss_acc, loss);
      atomicAdd(d.ce.loss_acc + 1, 1.f);
    }
    if (d.ce.row_loss) d.ce.row_loss[row] = loss;
  }
  __syncthreads();
  if (!d.ce.write_grad) return;
  const float lse = bcast;
  const float scale = ignored ? 0.f : (d.ce.scale_ptr ? *d.ce.scale_ptr : 1.f) * d.ce.scale_mul;
  const float pmul = 1.f + 2.f * d.ce.zloss * lse;
  const float off = d.ce.smoothing / (float)d.V_total;
  const int64_t tgt = tg - d.v0;
  const int nvec = d.ce.V / 8;
  for (int i = threadIdx.x; i < nvec; i += THREADS) {
    uint4 v = reinterpret_cast<const uint4*>(z)[i];
    uint32_t vw[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 a = unpack_bf16x2(vw[e]);
      const int j0 = i * 8 + 2 * e;
      float g0 = __expf(a.x - lse) * pmul - off;
      float g1 = __expf(a.y - lse) * pmul - off;
      if (j0 == tgt) g0 -= (1.f - d.ce.smoothing);
      if (j0 + 1 == tgt) g1 -= (1.f - d.ce.smoothing);
      vw[e] = pack_bf16x2(g0 * scale, g1 * scale);
    }
    reinterpret_cast<uint4*>(z)[i] = make_uint4(vw[0], vw[1], vw[2], vw[3]);
  }
}

}  // namespace lk

using namespace lk;

extern "C" int lk_cross_entropy_vp(const LkCeVpDesc* d, cudaStream_t s) {
  LK_REQUIRE(d->ce.V % 8 == 0 && d->ce.ld % 8 == 0, "cross_entropy_vp: V_local and ld must be multiples of 8");
  LK_REQUIRE(d->stats && d->peer_stats && d->world >= 1, "cross_entropy_vp: stats buffers");
  if (d->ce.T == 0) return 0;
  if (d->phase == 1) {
    ce_vp_stats_kernel<512><<<d->ce.T, 512, 0, s>>>(*d);
    return check_launch("cross_entropy_vp_stats");
  }
  ce_vp_finish_kernel<512><<<d->ce.T, 512, 0, s>>>(*d);
  return check_launch("cross_entropy_vp_finish");
}

extern "C" int lk_cross_entropy(const LkCeDesc* d, cudaStream_t s) {
  LK_REQUIRE(d->V % 8 == 0 && d->ld % 8 == 0, "cross_entropy: V and ld must be multiples of 8");
  if (d->T == 0) return 0;
  ce_kernel<512><<<d->T, 512, 0, s>>>((__nv_bfloat16*)d->logits, d->ld, d->targets, d->T, d->V,
                                      d->loss_acc, d->row_loss, d->scale_ptr, d->scale_mul,
                                      d->smoothing, d->zloss, d->ignore_index, d->write_grad);
  return check_launch("cross_entropy");
}
