// K11 fused AdamW over flat fp32 master weights, plus the single-GPU half of
// K12: gradient unscale + overflow check + global L2 norm, global-norm clip and
// the device-resident dynamic loss scaler.  No host synchronisation per step:
// every decision (skip the step, clip coefficient, new loss scale, bias
// correction step) lives in a small fp32 state vector on the device.
//
// Reference behaviour being re-implemented:
//   AdamW update   include/nn/training_pipeline.hpp:229-262 (decoupled wd:
//                  p -= lr*(wd*p + mhat/(sqrt(vhat)+eps)))
//   clipping       include/nn/optimizer_and_loss.hpp:34-56 (here global-norm)
//   loss scaling   include/nn/loss_scaling.hpp:8-53 (init 65536, x2 after
//                  2000 clean steps, /2 on overflow, floor 1)
//   health         include/nn/gradient_health.hpp:11-85 (skip on NaN/Inf;
//                  here the consecutive-skip counter resets on a good step)
//   EMA            include/nn/training_enhancements.hpp:124-142
#include "common.cuh"
#include "host_util.h"
#include "lk_api.h"

namespace lk {

// Chunk table entry: [start, length, weight-decay on/off, unused]
__global__ void __launch_bounds__(256) adamw_kernel(float* __restrict__ p32, float* __restrict__ g,
                                                    float* __restrict__ m, float* __restrict__ v,
                                                    __nv_bfloat16* __restrict__ p16,
                                                    float* __restrict__ ema,
                                                    const int4* __restrict__ chunks,
                                                    const float* __restrict__ state, float beta1,
                                                    float beta2, float eps, float wd,
                                                    float ema_decay, int zero_grad,
                                                    __nv_bfloat16* const* __restrict__ p16_peers,
                                                    int world) {
  if (state[LK_ST_SKIP] != 0.f) {
    // overflow step: only clear the gradient
    if (zero_grad) {
      const int4 ck = chunks[blockIdx.x];
      for (int i = threadIdx.x; i < ck.y; i += blockDim.x) g[ck.x + i] = 0.f;
    }
    return;
  }
  const int4 ck = chunks[blockIdx.x];
  const float lr = state[LK_ST_LR];
  const float gm = state[LK_ST_GRAD_MULT];
  const float step = state[LK_ST_STEP];
  const float bc1 = 1.f - powf(beta1, step);
  const float bc2 = 1.f - powf(beta2, step);
  const float wdl = ck.z ? wd : 0.f;
  const int64_t base = ck.x;
  const int n4 = ck.y / 4;
  for (int i = threadIdx.x; i < n4; i += blockDim.x) {
    const int64_t o = base + 4 * (int64_t)i;
    float4 P = *reinterpret_cast<float4*>(p32 + o);
    float4 G = *reinterpret_cast<float4*>(g + o);
    float4 Mm = *reinterpret_cast<float4*>(m + o);
    float4 Vv = *reinterpret_cast<float4*>(v + o);
    float* pp = &P.x;
    float* gg = &G.x;
    float* mm = &Mm.x;
    float* vv = &Vv.x;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float gr = gg[e] * gm;
      mm[e] = beta1 * mm[e] + (1.f - beta1) * gr;
      vv[e] = beta2 * vv[e] + (1.f - beta2) * gr * gr;
      const float mh = mm[e] / bc1;
      const float vh = vv[e] / bc2;
      pp[e] = pp[e] - lr * (wdl * pp[e] + mh / (sqrtf(vh) + eps));
    }
    *reinterpret_cast<float4*>(p32 + o) = P;
    *reinterpret_cast<float4*>(m + o) = Mm;
    *reinterpret_cast<float4*>(v + o) = Vv;
    if (zero_grad) *reinterpret_cast<float4*>(g + o) = make_float4(0.f, 0.f, 0.f, 0.f);
    const uint2 pb = make_uint2(pack_bf16x2(P.x, P.y), pack_bf16x2(P.z, P.w));
    if (p16) *reinterpret_cast<uint2*>(p16 + o) = pb;
    if (p16_peers) {
      const int64_t fo = o + 64 * (int64_t)ck.w;
      for (int q = 0; q < world; ++q) *reinterpret_cast<uint2*>(p16_peers[q] + fo) = pb;
    }
    if (ema) {
      float4 E = *reinterpret_cast<float4*>(ema + o);
      E.x = ema_decay * E.x + (1.f - ema_decay) * P.x;
      E.y = ema_decay * E.y + (1.f - ema_decay) * P.y;
      E.z = ema_decay * E.z + (1.f - ema_decay) * P.z;
      E.w = ema_decay * E.w + (1.f - ema_decay) * P.w;
      *reinterpret_cast<float4*>(ema + o) = E;
    }
  }
  // scalar tail (chunk lengths are multiples of 4 in practice)
  for (int i = 4 * n4 + threadIdx.x; i < ck.y; i += blockDim.x) {
    const int64_t o = base + i;
    const float gr = g[o] * gm;
    m[o] = beta1 * m[o] + (1.f - beta1) * gr;
    v[o] = beta2 * v[o] + (1.f - beta2) * gr * gr;
    p32[o] = p32[o] - lr * (wdl * p32[o] + (m[o] / bc1) / (sqrtf(v[o] / bc2) + eps));
    if (zero_grad) g[o] = 0.f;
    if (p16) p16[o] = __float2bfloat16(p32[o]);
    if (p16_peers)
      for (int q = 0; q < world; ++q) p16_peers[q][o + 64 * (int64_t)ck.w] = __float2bfloat16(p32[o]);
    if (ema) ema[o] = ema_decay * ema[o] + (1.f - ema_decay) * p32[o];
  }
}

// Per-block partial sum of squares of g (fp32) and a non-finite flag.
__global__ void __launch_bounds__(256) sumsq_kernel(const float* __restrict__ g, int64_t n,
                                                    float* __restrict__ partial) {
  __shared__ float red[8];
  float s = 0.f;
  const int64_t n4 = n / 4;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float4 a = reinterpret_cast<const float4*>(g)[i];
    s += a.x * a.x + a.y * a.y + a.z * a.z + a.w * a.w;
  }
  if (blockIdx.x == 0)
    for (int64_t i = 4 * n4 + threadIdx.x; i < n; i += blockDim.x) s += g[i] * g[i];
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int k = 0; k < 8; ++k) t += red[k];
    partial[blockIdx.x] = t;  // inf/nan propagate: overflow shows up here
  }
}

// Reduce the partials, set skip/clip/loss-scale/step in the state vector.
__global__ void finalize_kernel(const float* __restrict__ partial, int nparts, float* state,
                                float max_norm, int dynamic, float growth, float backoff,
                                int growth_interval, float min_scale) {
  __shared__ double red[256];
  double s = 0.0;
  for (int i = threadIdx.x; i < nparts; i += blockDim.x) s += (double)partial[i];
  red[threadIdx.x] = s;
  __syncthreads();
  for (int o = blockDim.x / 2; o > 0; o >>= 1) {
    if (threadIdx.x < o) red[threadIdx.x] += red[threadIdx.x + o];
    __syncthreads();
  }
  if (threadIdx.x != 0) return;
  const double tot = red[0];
  const float scale = state[LK_ST_LOSS_SCALE];
  const bool overflow = !isfinite(tot);
  const float norm = overflow ? INFINITY : (float)(sqrt(tot) / (double)scale);
  state[LK_ST_GRAD_NORM] = norm;
  if (overflow) {
    state[LK_ST_SKIP] = 1.f;
    state[LK_ST_NUM_SKIPPED] += 1.f;
    state[LK_ST_CONSEC_SKIPS] += 1.f;
    if (dynamic) state[LK_ST_LOSS_SCALE] = fmaxf(scale * backoff, min_scale);
    state[LK_ST_GROWTH_TRACKER] = 0.f;
    return;
  }
  const float clip = (max_norm > 0.f && norm > max_norm) ? max_norm / (norm + 1e-6f) : 1.f;
  state[LK_ST_CLIP_COEF] = clip;
  state[LK_ST_GRAD_MULT] = clip / scale;
  state[LK_ST_SKIP] = 0.f;
  state[LK_ST_CONSEC_SKIPS] = 0.f;
  state[LK_ST_STEP] += 1.f;
  if (dynamic) {
    const float t = state[LK_ST_GROWTH_TRACKER] + 1.f;
    if (t >= (float)growth_interval) {
      state[LK_ST_LOSS_SCALE] = scale * growth;
      state[LK_ST_GROWTH_TRACKER] = 0.f;
    } else {
      state[LK_ST_GROWTH_TRACKER] = t;
    }
  }
}

}  // namespace lk

using namespace lk;

extern "C" int lk_grad_norm_partials(const float* g, int64_t n, float* partial, int nparts,
                                     cudaStream_t s) {
  LK_REQUIRE(nparts > 0, "grad_norm: need partial slots");
  sumsq_kernel<<<nparts, 256, 0, s>>>(g, n, partial);
  return check_launch("sumsq");
}

extern "C" int lk_optimizer_finalize(const float* partial, int nparts, float* state,
                                     float max_norm, int dynamic, float growth, float backoff,
                                     int growth_interval, float min_scale, cudaStream_t s) {
  finalize_kernel<<<1, 256, 0, s>>>(partial, nparts, state, max_norm, dynamic, growth, backoff,
                                     growth_interval, min_scale);
  return check_launch("optimizer_finalize");
}

extern "C" int lk_adamw(const LkAdamWDesc* d, cudaStream_t s) {
  if (d->nchunks == 0) return 0;
  adamw_kernel<<<d->nchunks, 256, 0, s>>>(d->p32, d->g, d->m, d->v, (__nv_bfloat16*)d->p16, d->ema,
                                          (const int4*)d->chunks, d->state, d->beta1, d->beta2,
                                          d->eps, d->wd, d->ema_decay, d->zero_grad,
                                          (__nv_bfloat16* const*)d->p16_peers, d->world);
  return check_launch("adamw");
}
