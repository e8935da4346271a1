// K6 RoPE, K7 SwiGLU backward and K8 embedding gather / scatter-add.
//
// RoPE uses the reference's interleaved-pair convention (dims (2i, 2i+1) of a
// head rotate together, theta_i = pos * base^(-2i/head_dim);
// include/core/tensor.hpp:466-500) but per head with head_dim = Dh, not over
// the whole hidden width as src/nn/transformer_blocks.cpp:40-44 does.  The
// cos/sin table is computed on the host in float64 and passed in as float2.
//
// SwiGLU: h = silu(g) * u (forward fused into the gate|up GEMM epilogue);
// the backward here reads the stored gate|up tile layout (blocks of 128 gate
// columns followed by 128 up columns) and writes d(gate|up) in the same layout.
// Reference: swiglu_forward/backward include/core/tensor.hpp:440-458.
//
// Embedding: the reference never produces embedding gradients
// (src/nn/transformer_blocks.cpp:670-718); here the backward scatter-adds into
// the fp32 gradient with vector atomics.  Out-of-range token ids are recorded
// in the status word and read as a zero row instead of faulting.
#include <algorithm>

#include "common.cuh"
#include "host_util.h"
#include "lk_api.h"

namespace lk {

// ------------------------------------------------------------------ RoPE
// x: [T, ncols] bf16 (row pitch ld); heads [0, nheads) of width Dh starting at
// column col0 are rotated in place.  pos[t] gives the position of token t (or
// t % seq_len + pos_offset when pos == nullptr).  inverse != 0 applies the
// inverse rotation (backward).
__global__ void rope_kernel(__nv_bfloat16* __restrict__ x, int64_t ld, int T, int col0,
                            int nheads, int Dh, const float2* __restrict__ table,
                            const int* __restrict__ pos, int seq_len, int pos_offset,
                            int inverse) {
  const int vec_per_head = Dh / 8;  // 8 bf16 = 4 rotation pairs per thread
  const int64_t total = (int64_t)T * nheads * vec_per_head;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int v = (int)(idx % vec_per_head);
    const int64_t th = idx / vec_per_head;
    const int h = (int)(th % nheads);
    const int t = (int)(th / nheads);
    const int p = pos ? pos[t] : (t % seq_len) + pos_offset;
    uint4* ptr = reinterpret_cast<uint4*>(x + (int64_t)t * ld + col0 + h * Dh + v * 8);
    uint4 a = *ptr;
    uint32_t w[4] = {a.x, a.y, a.z, a.w};
    const float2* tb = table + (int64_t)p * (Dh / 2) + v * 4;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 cs = tb[e];
      const float s = inverse ? -cs.y : cs.y;
      const float2 f = unpack_bf16x2(w[e]);
      w[e] = pack_bf16x2(f.x * cs.x - f.y * s, f.x * s + f.y * cs.x);
    }
    *ptr = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// --------------------------------------------------------------- SwiGLU bwd
__device__ __forceinline__ float sigmoid_f(float x) { return 1.0f / (1.0f + __expf(-x)); }

__global__ void swiglu_bwd_kernel(const __nv_bfloat16* __restrict__ gu,
                                  const __nv_bfloat16* __restrict__ dh,
                                  __nv_bfloat16* __restrict__ dgu, int M, int F) {
  const int vec_per_row = F / 8;
  const int64_t total = (int64_t)M * vec_per_row;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int row = (int)(idx / vec_per_row);
    const int c = (int)(idx % vec_per_row) * 8;  // column in h
    const int blk = c >> 7, off = c & 127;
    const int64_t gcol = (int64_t)blk * 256 + off;
    const int64_t base = (int64_t)row * 2 * F;
    const uint4 gv = *reinterpret_cast<const uint4*>(gu + base + gcol);
    const uint4 uv = *reinterpret_cast<const uint4*>(gu + base + gcol + 128);
    const uint4 hv = *reinterpret_cast<const uint4*>(dh + (int64_t)row * F + c);
    const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w};
    const uint32_t uw[4] = {uv.x, uv.y, uv.z, uv.w};
    const uint32_t hw[4] = {hv.x, hv.y, hv.z, hv.w};
    uint32_t dg[4], du[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 g = unpack_bf16x2(gw[e]), u = unpack_bf16x2(uw[e]), d = unpack_bf16x2(hw[e]);
      const float s0 = sigmoid_f(g.x), s1 = sigmoid_f(g.y);
      const float si0 = g.x * s0, si1 = g.y * s1;
      dg[e] = pack_bf16x2(d.x * u.x * s0 * (1.f + g.x * (1.f - s0)),
                          d.y * u.y * s1 * (1.f + g.y * (1.f - s1)));
      du[e] = pack_bf16x2(d.x * si0, d.y * si1);
    }
    *reinterpret_cast<uint4*>(dgu + base + gcol) = make_uint4(dg[0], dg[1], dg[2], dg[3]);
    *reinterpret_cast<uint4*>(dgu + base + gcol + 128) = make_uint4(du[0], du[1], du[2], du[3]);
  }
}

// Plain forward (h = silu(g)*u from the same gate|up layout), for callers that
// did not fuse it into the GEMM epilogue.
__global__ void swiglu_fwd_kernel(const __nv_bfloat16* __restrict__ gu,
                                  __nv_bfloat16* __restrict__ h, int M, int F) {
  const int vec_per_row = F / 8;
  const int64_t total = (int64_t)M * vec_per_row;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int row = (int)(idx / vec_per_row);
    const int c = (int)(idx % vec_per_row) * 8;
    const int64_t gcol = (int64_t)(c >> 7) * 256 + (c & 127);
    const int64_t base = (int64_t)row * 2 * F;
    const uint4 gv = *reinterpret_cast<const uint4*>(gu + base + gcol);
    const uint4 uv = *reinterpret_cast<const uint4*>(gu + base + gcol + 128);
    const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w};
    const uint32_t uw[4] = {uv.x, uv.y, uv.z, uv.w};
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 g = unpack_bf16x2(gw[e]), u = unpack_bf16x2(uw[e]);
      o[e] = pack_bf16x2(g.x * sigmoid_f(g.x) * u.x, g.y * sigmoid_f(g.y) * u.y);
    }
    *reinterpret_cast<uint4*>(h + (int64_t)row * F + c) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// -------------------------------------------------------------- embedding
__global__ void embed_fwd_kernel(const int64_t* __restrict__ ids, const __nv_bfloat16* __restrict__ W,
                                 __nv_bfloat16* __restrict__ out, int T, int D, int V, int* status) {
  const int vec = D / 8;
  const int64_t total = (int64_t)T * vec;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int t = (int)(idx / vec), c = (int)(idx % vec);
    const int64_t id = ids[t];
    uint4 v = make_uint4(0, 0, 0, 0);
    if (id >= 0 && id < V)
      v = reinterpret_cast<const uint4*>(W + id * D)[c];
    else if (c == 0 && status)
      atomicCAS(status, 0, LK_ERR_BAD_INDEX);
    reinterpret_cast<uint4*>(out + (int64_t)t * D)[c] = v;
  }
}

__global__ void embed_bwd_kernel(const int64_t* __restrict__ ids, const __nv_bfloat16* __restrict__ dy,
                                 float* __restrict__ dW, int T, int D, int V) {
  const int vec = D / 4;
  const int64_t total = (int64_t)T * vec;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int t = (int)(idx / vec), c = (int)(idx % vec);
    const int64_t id = ids[t];
    if (id < 0 || id >= V) continue;
    const uint2 g = reinterpret_cast<const uint2*>(dy + (int64_t)t * D)[c];
    const float2 a = unpack_bf16x2(g.x), b = unpack_bf16x2(g.y);
    atomicAdd(reinterpret_cast<float4*>(dW + id * D) + c, make_float4(a.x, a.y, b.x, b.y));
  }
}

static int grid_for(int64_t work, int threads) {
  int64_t g = (work + threads - 1) / threads;
  const int64_t cap = (int64_t)num_sms() * 16;
  if (g > cap) g = cap;
  return (int)(g < 1 ? 1 : g);
}

}  // namespace lk

using namespace lk;

// fp32 -> bf16, 8 elements per thread (the vocabulary-chunked LM head sums its
// input gradient over chunks in fp32 and rounds once)
__global__ void cast_f32_bf16_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ y, int64_t n8) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
    const float4 a = reinterpret_cast<const float4*>(x)[2 * i];
    const float4 b = reinterpret_cast<const float4*>(x)[2 * i + 1];
    reinterpret_cast<uint4*>(y)[i] = make_uint4(pack_bf16x2(a.x, a.y), pack_bf16x2(a.z, a.w),
                                                pack_bf16x2(b.x, b.y), pack_bf16x2(b.z, b.w));
  }
}

extern "C" int lk_cast_f32_bf16(const float* x, void* y, int64_t n, cudaStream_t s) {
  LK_REQUIRE(n % 8 == 0 && ((uintptr_t)x & 15) == 0 && ((uintptr_t)y & 15) == 0,
             "cast_f32_bf16: n % 8 == 0 and 16-byte aligned buffers");
  if (n == 0) return 0;
  const int64_t n8 = n / 8;
  int grid = (int)std::min<int64_t>((n8 + 255) / 256, (int64_t)num_sms() * 8);
  cast_f32_bf16_kernel<<<grid, 256, 0, s>>>(x, (__nv_bfloat16*)y, n8);
  return check_launch("cast_f32_bf16");
}

extern "C" int lk_rope(const LkRopeDesc* d, cudaStream_t s) {
  LK_REQUIRE(d->Dh % 8 == 0 && d->col0 % 8 == 0 && d->ld % 8 == 0, "rope: head_dim/col0/ld must be multiples of 8");
  const int64_t work = (int64_t)d->T * d->nheads * (d->Dh / 8);
  if (work == 0) return 0;
  rope_kernel<<<grid_for(work, 256), 256, 0, s>>>((__nv_bfloat16*)d->x, d->ld, d->T, d->col0,
                                                   d->nheads, d->Dh, (const float2*)d->table, d->pos,
                                                   d->seq_len, d->pos_offset, d->inverse);
  return check_launch("rope");
}

extern "C" int lk_swiglu_bwd(const void* gu, const void* dh, void* dgu, int M, int F,
                             cudaStream_t s) {
  LK_REQUIRE(F % 128 == 0, "swiglu_bwd: F must be a multiple of 128");
  swiglu_bwd_kernel<<<grid_for((int64_t)M * F / 8, 256), 256, 0, s>>>(
      (const __nv_bfloat16*)gu, (const __nv_bfloat16*)dh, (__nv_bfloat16*)dgu, M, F);
  return check_launch("swiglu_bwd");
}

extern "C" int lk_swiglu_fwd(const void* gu, void* h, int M, int F, cudaStream_t s) {
  LK_REQUIRE(F % 128 == 0, "swiglu_fwd: F must be a multiple of 128");
  swiglu_fwd_kernel<<<grid_for((int64_t)M * F / 8, 256), 256, 0, s>>>(
      (const __nv_bfloat16*)gu, (__nv_bfloat16*)h, M, F);
  return check_launch("swiglu_fwd");
}

extern "C" int lk_embedding_fwd(const int64_t* ids, const void* W, void* out, int T, int D, int V,
                                int* status, cudaStream_t s) {
  LK_REQUIRE(D % 8 == 0, "embedding: D must be a multiple of 8");
  embed_fwd_kernel<<<grid_for((int64_t)T * D / 8, 256), 256, 0, s>>>(
      ids, (const __nv_bfloat16*)W, (__nv_bfloat16*)out, T, D, V, status);
  return check_launch("embedding_fwd");
}

extern "C" int lk_embedding_bwd(const int64_t* ids, const void* dy, float* dW, int T, int D, int V,
                                cudaStream_t s) {
  LK_REQUIRE(D % 4 == 0, "embedding_bwd: D must be a multiple of 4");
  embed_bwd_kernel<<<grid_for((int64_t)T * D / 4, 256), 256, 0, s>>>(
      ids, (const __nv_bfloat16*)dy, dW, T, D, V);
  return check_launch("embedding_bwd");
}
