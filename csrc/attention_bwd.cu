// K4: flash-attention backward on tcgen05 (causal / full / sliding window, GQA,
// head_dim 64/128).
//
// One CTA per (128-key tile j, kv head g, batch b).  It loops over every q head
// of the GQA group and every q tile i that can see key tile j, so dK_j and dV_j
// accumulate in TMEM for the whole group and are written once (no atomics):
//
//   S^T  = K_j Q_i^T            (tcgen05, M = keys, N = queries)
//   dP^T = V_j dO_i^T
//   P^T  = exp(S^T * scale - LSE),  dS^T = P^T (dP^T - D) * scale   (registers)
//   dV  += P^T dO_i,  dK += dS^T Q_i,  dQ_i = dS K_j                 (tcgen05)
//
// dQ_i partials go from TMEM through a shared-memory staging tile into the fp32
// accumulator with bulk tensor reduce-adds (cp.reduce.async.bulk.tensor, whole
// 128-byte lines, no multicast) and are converted to bf16 by a final kernel.  The same
// 128B-swizzled shared-memory tiles serve as K-major operands (S^T, dP^T) and
// as MN-major operands (dV, dK, dQ), so nothing is transposed in memory.
// D = rowsum(dO * O) is computed by a small pre-pass, which also zeroes the
// fp32 dQ accumulator.
//
// Replaces the reference's MultiHeadAttention::backward
// (src/nn/transformer_blocks.cpp:156-207) and softmax_backward_inplace
// (include/core/tensor.hpp:380-392).
#include "common.cuh"
#include "host_util.h"
#include "lk_api.h"

namespace lk {

// element offset of the LSE * log2(e) half of the dvec scratch (16-byte aligned)
static inline int64_t lk_attn_dvec_half(int B, int Hq, int S) {
  return ((int64_t)B * Hq * S + 63) / 64 * 64;
}

struct AttnBwdArgs {
  int B, S, Hq, Hkv;
  int causal, window;
  float sl2;    // scale * log2(e)
  float scale;  // softmax scale
  const float* lse;   // [B, Hq, S] LSE * log2(e)
  const float* Dvec;  // [B, Hq, S] scale * rowsum(dO * O)
  float* dq_acc;      // [B*S, Hq*Dh] fp32
  __nv_bfloat16* dqkv;
  int64_t ld_dqkv;
  int* status;
  int n_tiles;
};

__device__ __forceinline__ uint32_t sw128_off_b(int r, int u) {
  return (uint32_t)((u >> 3) * 16384 + r * 128 + (((u & 7) ^ (r & 7)) << 4));
}

// head_dim 64: P^T lives in its own TMEM columns and is the A operand of the
// dV MMA (no shared-memory round trip), and the skewed schedule runs S^T/dP^T of
// iteration it+1 before the gradient MMAs of it.  head_dim 128 has no TMEM
// left for either (dQ reuses S^T's columns): P goes through shared memory and
// the schedule is serial.
template <int DH>
struct BwdCfg {
  static constexpr bool P_TMEM = DH == 64;
  static constexpr int QB = 128 * DH * 2;
  static constexpr int STAGES = DH == 64 ? 3 : 1;
  static constexpr int NSW = DH == 64 ? 16 : 8;  // softmax warps
  static constexpr int NDRAIN = 8;  // warps that drain dQ (one 4 KB staging tile each)
  static constexpr int OFF_K = 0;
  static constexpr int OFF_V = QB;
  static constexpr int OFF_Q = 2 * QB;
  static constexpr int OFF_DO = OFF_Q + STAGES * QB;
  static constexpr int OFF_DS = OFF_DO + STAGES * QB;
  static constexpr int OFF_P = OFF_DS + 32768;                     // unused when P_TMEM
  static constexpr int OFF_STG = OFF_P + (P_TMEM ? 0 : 32768);     // dQ staging, 1024-aligned
  static constexpr int OFF_LD = OFF_STG + NDRAIN * 4096;           // [STAGES][2][128] fp32 LSE, D
  static constexpr int OFF_BAR = OFF_LD + STAGES * 1024;
  static constexpr int SMEM = OFF_BAR + 256;
  static constexpr int TMEM_COLS = 512;
};

__device__ __forceinline__ void q_range(const AttnBwdArgs& a, int j, int& i0, int& i1) {
  const int n = a.n_tiles;
  i0 = a.causal ? j : 0;
  i1 = n;
  if (a.window > 0) {
    // query q sees keys in (q - window, q]; key tile j is seen by q < j*128 + 127 + window
    const int qmax = j * 128 + 127 + a.window - 1;
    i1 = min(n, qmax / 128 + 1);
  }
}

template <int DH>
constexpr int bwd_softmax_warps() { return BwdCfg<DH>::NSW; }

template <int DH>
__global__ void __launch_bounds__(64 + 32 * bwd_softmax_warps<DH>(), 1)
    attn_bwd_kernel(const __grid_constant__ CUtensorMap tm_qkv, const __grid_constant__ CUtensorMap tm_do,
                    const __grid_constant__ CUtensorMap tm_dq, const AttnBwdArgs args) {
  using C = BwdCfg<DH>;
  constexpr bool P_TMEM = C::P_TMEM;
  constexpr bool SKEW = P_TMEM;       // needs dQ in its own TMEM columns
  constexpr bool DQ_ALIAS = !P_TMEM;  // head_dim 128: dQ reuses S^T's columns
  constexpr int NSW = C::NSW;
  constexpr int NG = NSW / 4;   // warps per TMEM lane quarter
  constexpr int CPW = 4 / NG;   // 32-query chunks per warp
  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t sbase = smem_u32(smem);
  if (sbase & 1023) {
    if (threadIdx.x == 0) atomicCAS(args.status, 0, LK_ERR_BAD_INDEX);
    return;
  }
  const uint32_t bar = sbase + C::OFF_BAR;
  const uint32_t kv_full = bar, qd_full = bar + 8, qd_empty = bar + 32, sdp_full = bar + 56,
                 sdp_free = bar + 64, ds_ready = bar + 72, dq_full = bar + 80, dq_free = bar + 88,
                 drain = bar + 96, pds_free = bar + 104;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_BAR + 128);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_BAR + 132);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // 1-D grid, key tile slowest: all j = 0 CTAs (the most work when causal) first
  const int gb = args.Hkv * args.B;
  const int j = (int)(blockIdx.x / gb);
  const int g = (int)(blockIdx.x % gb) % args.Hkv, b = (int)(blockIdx.x % gb) / args.Hkv;
  const int group = args.Hq / args.Hkv;
  const int S = args.S;
  const int row0 = b * S;
  int i0, i1;
  q_range(args, j, i0, i1);
  const int nq = max(0, i1 - i0);
  const int n_it = group * nq;
  // whole 128-query tiles: LSE/D rows arrive by bulk copy with the Q/dO stage
  const bool bulk_ld = (S & 127) == 0;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int s2 = 0; s2 < C::STAGES; ++s2) {
      mbar_init(qd_full + 8 * s2, 1);
      mbar_init(qd_empty + 8 * s2, 1);
    }
    mbar_init(pds_free, 1);
    mbar_init(sdp_full, 1);
    mbar_init(sdp_free, NSW);
    mbar_init(ds_ready, NSW);
    mbar_init(dq_full, 1);
    mbar_init(dq_free, NSW);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tm_qkv);
    tma_prefetch_desc(&tm_do);
    tma_prefetch_desc(&tm_dq);
  }
  if (warp == 1) tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem, tdP = tmem + 128, tdV = tmem + 256, tdK = tmem + 256 + DH;
  const uint32_t tdQ = DQ_ALIAS ? tS : tmem + 256 + 2 * DH;
  const uint32_t tP = tmem + 256 + 3 * DH;  // P^T, bf16 pairs (head_dim 64 only)

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ TMA
      mbar_expect_tx(kv_full, 2 * C::QB);
#pragma unroll
      for (int c = 0; c < DH / 64; ++c) {
        tma_load_2d(sbase + C::OFF_K + c * 16384, &tm_qkv, kv_full, (args.Hq + g) * DH + c * 64, row0 + j * 128);
        tma_load_2d(sbase + C::OFF_V + c * 16384, &tm_qkv, kv_full,
                    (args.Hq + args.Hkv + g) * DH + c * 64, row0 + j * 128);
      }
      uint32_t pending = 0, parbits = 0;
      bool ok = true;
      for (int it = 0; it < n_it && ok; ++it) {
        const int h = g * group + it / nq;
        const int i = i0 + it % nq;
        const int st = it % C::STAGES;
        const uint32_t ph = (uint32_t)(it / C::STAGES) & 1;
        if (!bounded_wait(qd_empty + 8 * st, ph ^ 1, args.status, LK_ERR_TIMEOUT_EMPTY, abort_flag)) {
          ok = false;
          break;
        }
        const uint32_t fb = qd_full + 8 * st;
        mbar_expect_tx(fb, 2 * C::QB + (bulk_ld ? 1024u : 0u));
        if (bulk_ld) {
          const int64_t off = ((int64_t)b * args.Hq + h) * S + i * 128;
          bulk_load(sbase + C::OFF_LD + st * 1024, args.lse + off, 512, fb);
          bulk_load(sbase + C::OFF_LD + st * 1024 + 512, args.Dvec + off, 512, fb);
        }
#pragma unroll
        for (int c = 0; c < DH / 64; ++c) {
          tma_load_2d(sbase + C::OFF_Q + st * C::QB + c * 16384, &tm_qkv, fb, h * DH + c * 64, row0 + i * 128);
          tma_load_2d(sbase + C::OFF_DO + st * C::QB + c * 16384, &tm_do, fb, h * DH + c * 64, row0 + i * 128);
        }
        pending |= 1u << st;
        parbits = (parbits & ~(1u << st)) | (ph << st);
      }
      if (!ok) {
        bounded_wait(kv_full, 0, args.status, LK_ERR_TIMEOUT_DRAIN, nullptr);
        for (int s2 = 0; s2 < C::STAGES; ++s2)
          if (pending & (1u << s2))
            bounded_wait(qd_full + 8 * s2, (parbits >> s2) & 1, args.status, LK_ERR_TIMEOUT_DRAIN, nullptr);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------ MMA
      constexpr uint32_t id_s = make_idesc_bf16(128, 128, false, false);   // K Q^T, V dO^T
      constexpr uint32_t id_kv = make_idesc_bf16(128, DH, false, true);    // P^T dO, dS^T Q
      constexpr uint32_t id_q = make_idesc_bf16(128, DH, true, true);      // dS K
      const uint32_t sk = sbase + C::OFF_K, sv = sbase + C::OFF_V;
      const uint32_t sp = sbase + C::OFF_P, sds = sbase + C::OFF_DS;
      bool ok = bounded_wait(kv_full, 0, args.status, LK_ERR_TIMEOUT_FULL, abort_flag);
      auto issue_sdp = [&](int it) {
        const int st = it % C::STAGES;
        const uint32_t sq = sbase + C::OFF_Q + st * C::QB, sdo = sbase + C::OFF_DO + st * C::QB;
#pragma unroll
        for (int kk = 0; kk < DH / 16; ++kk) {
          const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
          tc_mma_f16(tS, make_desc_sw128(sk + off, 16, 1024), make_desc_sw128(sq + off, 16, 1024), id_s,
                     kk > 0 ? 1u : 0u);
        }
#pragma unroll
        for (int kk = 0; kk < DH / 16; ++kk) {
          const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
          tc_mma_f16(tdP, make_desc_sw128(sv + off, 16, 1024), make_desc_sw128(sdo + off, 16, 1024), id_s,
                     kk > 0 ? 1u : 0u);
        }
        tc_commit(sdp_full);
      };
      // gradient MMAs of iteration m: dV += P^T dO, dK += dS^T Q, dQ = dS K
      auto issue_grad = [&](int m) {
        const int stm = m % C::STAGES;
        const uint32_t sq = sbase + C::OFF_Q + stm * C::QB, sdo = sbase + C::OFF_DO + stm * C::QB;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {  // contraction over the 128 queries
          const uint32_t aoff = (kk >> 2) * 16384 + (kk & 3) * 32;
          if constexpr (P_TMEM)
            tc_mma_f16_ta(tdV, tP + kk * 8, make_desc_sw128(sdo + kk * 2048, 16384, 1024), id_kv,
                          (m > 0 || kk > 0) ? 1u : 0u);
          else
            tc_mma_f16(tdV, make_desc_sw128(sp + aoff, 16, 1024), make_desc_sw128(sdo + kk * 2048, 16384, 1024),
                       id_kv, (m > 0 || kk > 0) ? 1u : 0u);
          tc_mma_f16(tdK, make_desc_sw128(sds + aoff, 16, 1024), make_desc_sw128(sq + kk * 2048, 16384, 1024),
                     id_kv, (m > 0 || kk > 0) ? 1u : 0u);
        }
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)  // contraction over the 128 keys
          tc_mma_f16(tdQ, make_desc_sw128(sds + kk * 2048, 16384, 1024),
                     make_desc_sw128(sk + kk * 2048, 16384, 1024), id_q, kk > 0 ? 1u : 0u);
        tc_commit(dq_full);
        tc_commit(qd_empty + 8 * stm);
        tc_commit(pds_free);
      };
      for (int it = 0; it < n_it && ok; ++it) {
        const int st = it % C::STAGES;
        const uint32_t ph = (uint32_t)(it / C::STAGES) & 1;
        const uint32_t prev = (uint32_t)(it - 1) & 1;
        if (!bounded_wait(qd_full + 8 * st, ph, args.status, LK_ERR_TIMEOUT_FULL, abort_flag) ||
            (it > 0 && !bounded_wait(sdp_free, prev, args.status, LK_ERR_TIMEOUT_ACCUM, abort_flag)) ||
            (DQ_ALIAS && it > 0 && !bounded_wait(dq_free, prev, args.status, LK_ERR_TIMEOUT_ACCUM, abort_flag))) {
          ok = false;
          break;
        }
        tc_fence_after();
        issue_sdp(it);
        // skewed: the gradient MMAs of it-1 follow S^T/dP^T of it; serial: those of it
        const int m = SKEW ? it - 1 : it;
        if (m >= 0) {
          if (!bounded_wait(ds_ready, m & 1, args.status, LK_ERR_TIMEOUT_ACCUM, abort_flag) ||
              (!DQ_ALIAS && m > 0 && !bounded_wait(dq_free, (m - 1) & 1, args.status, LK_ERR_TIMEOUT_ACCUM, abort_flag))) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_grad(m);
        }
      }
      if (SKEW && ok && n_it > 0) {
        const int m = n_it - 1;
        if (bounded_wait(ds_ready, m & 1, args.status, LK_ERR_TIMEOUT_ACCUM, abort_flag) &&
            (m == 0 || bounded_wait(dq_free, (m - 1) & 1, args.status, LK_ERR_TIMEOUT_ACCUM, abort_flag))) {
          tc_fence_after();
          issue_grad(m);
        }
      }
      tc_commit(drain);
      bounded_wait(drain, 0, args.status, LK_ERR_TIMEOUT_DRAIN, nullptr);
    }
  } else {
    // ------------------------------------------------- softmax backward
    // warp w owns TMEM lanes 32*(w%4)..+31 (key rows of S^T/dP^T/dK/dV, query
    // rows of dQ) and query chunks wg*CPW .. +CPW-1 (32 queries each).
    const int quarter = warp & 3;
    const int wg = (warp - 2) >> 2;
    const int kr = quarter * 32 + lane;
    const int key = j * 128 + kr;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    uint8_t* sP = smem + C::OFF_P;
    uint8_t* sDS = smem + C::OFF_DS;
    // dQ staging: 32 rows x 32 fp32 columns (128B-swizzled) per draining warp
    // draining warps are those with wg < 2 (head_dim 64: chunks 0, 1; head_dim
    // 128: every warp, chunks wg and wg + 2): one tile per (quarter, wg)
    static_assert(C::NDRAIN == 8, "one staging tile per draining warp");
    const int drain_slot = (quarter * 2 + wg) & 7;
    const uint32_t stg = sbase + C::OFF_STG + drain_slot * 4096;
    uint8_t* stg_p = smem + C::OFF_STG + drain_slot * 4096;
    // dQ(m) from TMEM into the staging tile, then one bulk reduce-add into the
    // fp32 accumulator per 32 x 32 block
    auto drain_dq = [&](int m) {
      const int hm = g * group + m / nq;
      const int im = i0 + m % nq;
#pragma unroll 1
      for (int c = wg; c < DH / 32; c += NG) {
        uint32_t v[32];
        tmem_ld32(tdQ + lane_off + c * 32, v);
        tc_wait_ld();
        if (lane == 0) bulk_wait_read<0>();  // the previous reduce has read the staging tile
        __syncwarp();
#pragma unroll
        for (int u = 0; u < 8; ++u)
          *reinterpret_cast<uint4*>(stg_p + lane * 128 + ((u ^ (lane & 7)) << 4)) =
              make_uint4(v[4 * u], v[4 * u + 1], v[4 * u + 2], v[4 * u + 3]);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_reduce_add_2d(&tm_dq, stg, hm * DH + c * 32, row0 + im * 128 + quarter * 32);
          bulk_commit();
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(dq_free);
    };
    bool ok = true;
    for (int it = 0; it < n_it; ++it) {
      const int h = g * group + it / nq;
      const int i = i0 + it % nq;
      bool w_ok = bounded_wait(sdp_full, it & 1, args.status, LK_ERR_TIMEOUT_ACCUM, abort_flag);
      if (!__all_sync(0xffffffffu, w_ok)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const float* lse_row = args.lse + ((int64_t)b * args.Hq + h) * S + i * 128;
      const float* d_row = args.Dvec + ((int64_t)b * args.Hq + h) * S + i * 128;
      const bool need_mask = (args.causal && i == j) || (i + 1) * 128 > S || (j + 1) * 128 > S ||
                             args.window > 0;
      const bool vec_ok = (i * 128 + 127 < S) && (S & 3) == 0;
      const int st = it % C::STAGES;
      const float* sL = reinterpret_cast<const float*>(smem + C::OFF_LD + st * 1024);
      // P / dS of this warp's queries as bf16 pairs, built 16 queries at a time
      uint32_t pp[CPW][16], pd[CPW][16];
#pragma unroll
      for (int c = 0; c < CPW; ++c) {
        const int cc = wg * CPW + c;
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          uint32_t sv[16], dv[16];
          tmem_ld16(tS + lane_off + cc * 32 + hf * 16, sv);
          tmem_ld16(tdP + lane_off + cc * 32 + hf * 16, dv);
          tc_wait_ld();
          if (c == CPW - 1 && hf == 1) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(sdp_free);  // S^T / dP^T may be overwritten now
          }
#pragma unroll
          for (int e = 0; e < 16; e += 4) {
            const int qi = cc * 32 + hf * 16 + e;
            float Ls[4], Ds[4];
            if (bulk_ld) {
              const float4 L = *reinterpret_cast<const float4*>(sL + qi);
              const float4 Dd = *reinterpret_cast<const float4*>(sL + 128 + qi);
              Ls[0] = L.x; Ls[1] = L.y; Ls[2] = L.z; Ls[3] = L.w;
              Ds[0] = Dd.x; Ds[1] = Dd.y; Ds[2] = Dd.z; Ds[3] = Dd.w;
            } else if (vec_ok) {
              const float4 L = *reinterpret_cast<const float4*>(lse_row + qi);
              const float4 Dd = *reinterpret_cast<const float4*>(d_row + qi);
              Ls[0] = L.x; Ls[1] = L.y; Ls[2] = L.z; Ls[3] = L.w;
              Ds[0] = Dd.x; Ds[1] = Dd.y; Ds[2] = Dd.z; Ds[3] = Dd.w;
            } else {
#pragma unroll
              for (int t = 0; t < 4; ++t) {
                const bool in = i * 128 + qi + t < S;
                Ls[t] = in ? lse_row[qi + t] : 0.f;
                Ds[t] = in ? d_row[qi + t] : 0.f;
              }
            }
            float p[4], ds[4];
#pragma unroll
            for (int t = 0; t < 4; ++t) {
              const int q = i * 128 + qi + t;
              p[t] = fast_exp2(fmaf(__uint_as_float(sv[e + t]), args.sl2, -Ls[t]));
              if (need_mask && (q >= S || key >= S || (args.causal && key > q) ||
                                (args.window > 0 && key <= q - args.window)))
                p[t] = 0.f;
              ds[t] = p[t] * fmaf(__uint_as_float(dv[e + t]), args.scale, -Ds[t]);
            }
            pp[c][hf * 8 + e / 2] = pack_bf16x2(p[0], p[1]);
            pp[c][hf * 8 + e / 2 + 1] = pack_bf16x2(p[2], p[3]);
            pd[c][hf * 8 + e / 2] = pack_bf16x2(ds[0], ds[1]);
            pd[c][hf * 8 + e / 2 + 1] = pack_bf16x2(ds[2], ds[3]);
          }
        }
      }
      if (SKEW && it > 0) {
        // the gradient MMAs of it-1 are done: P^T / dS are free and dQ(it-1) is ready
        w_ok = bounded_wait(dq_full, (it - 1) & 1, args.status, LK_ERR_TIMEOUT_ACCUM, abort_flag) &&
               bounded_wait(pds_free, (it - 1) & 1, args.status, LK_ERR_TIMEOUT_ACCUM, abort_flag);
        if (!__all_sync(0xffffffffu, w_ok)) {
          ok = false;
          break;
        }
        tc_fence_after();
        drain_dq(it - 1);
      }
      if (!SKEW && it > 0) {
        // serial schedule: the previous gradient MMAs finished before dQ(it-1) was drained
        w_ok = bounded_wait(pds_free, (it - 1) & 1, args.status, LK_ERR_TIMEOUT_ACCUM, abort_flag);
        if (!__all_sync(0xffffffffu, w_ok)) {
          ok = false;
          break;
        }
        tc_fence_after();
      }
#pragma unroll
      for (int c = 0; c < CPW; ++c) {
        const int cc = wg * CPW + c;
        if constexpr (P_TMEM) {
          tmem_st16(tP + lane_off + cc * 16, pp[c]);
        } else {
#pragma unroll
          for (int u = 0; u < 4; ++u)
            *reinterpret_cast<uint4*>(sP + sw128_off_b(kr, cc * 4 + u)) =
                make_uint4(pp[c][4 * u], pp[c][4 * u + 1], pp[c][4 * u + 2], pp[c][4 * u + 3]);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u)
          *reinterpret_cast<uint4*>(sDS + sw128_off_b(kr, cc * 4 + u)) =
              make_uint4(pd[c][4 * u], pd[c][4 * u + 1], pd[c][4 * u + 2], pd[c][4 * u + 3]);
      }
      if constexpr (P_TMEM) tc_wait_st();
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(ds_ready);
      if (!SKEW) {
        w_ok = bounded_wait(dq_full, it & 1, args.status, LK_ERR_TIMEOUT_ACCUM, abort_flag);
        if (!__all_sync(0xffffffffu, w_ok)) {
          ok = false;
          break;
        }
        tc_fence_after();
        drain_dq(it);
      }
    }
    if (SKEW && ok && n_it > 0) {
      const bool w_ok = bounded_wait(dq_full, (n_it - 1) & 1, args.status, LK_ERR_TIMEOUT_ACCUM, abort_flag);
      if (__all_sync(0xffffffffu, w_ok)) {
        tc_fence_after();
        drain_dq(n_it - 1);
      } else {
        ok = false;
      }
    }
    // every bulk reduce of this warp has finished (its staging tile may go away)
    if (lane == 0) bulk_wait<0>();
    __syncwarp();
    // dK, dV (lane = key row) -> bf16 into dqkv.  tcgen05.ld is warp-collective:
    // every lane loads, only in-range keys store.
    if (__all_sync(0xffffffffu, ok) && n_it > 0) {
      tc_fence_after();
      __nv_bfloat16* dk = args.dqkv + (int64_t)(row0 + key) * args.ld_dqkv + (args.Hq + g) * DH;
      __nv_bfloat16* dvp = args.dqkv + (int64_t)(row0 + key) * args.ld_dqkv + (args.Hq + args.Hkv + g) * DH;
#pragma unroll 1
      for (int c = wg; c < DH / 32; c += NG) {
        uint32_t a[32], bb[32];
        tmem_ld32(tdK + lane_off + c * 32, a);
        tmem_ld32(tdV + lane_off + c * 32, bb);
        tc_wait_ld();
        if (key >= S) continue;
#pragma unroll
        for (int e = 0; e < 32; e += 8) {
          *reinterpret_cast<uint4*>(dk + c * 32 + e) = make_uint4(
              pack_bf16x2(__uint_as_float(a[e]), __uint_as_float(a[e + 1])),
              pack_bf16x2(__uint_as_float(a[e + 2]), __uint_as_float(a[e + 3])),
              pack_bf16x2(__uint_as_float(a[e + 4]), __uint_as_float(a[e + 5])),
              pack_bf16x2(__uint_as_float(a[e + 6]), __uint_as_float(a[e + 7])));
          *reinterpret_cast<uint4*>(dvp + c * 32 + e) = make_uint4(
              pack_bf16x2(__uint_as_float(bb[e]), __uint_as_float(bb[e + 1])),
              pack_bf16x2(__uint_as_float(bb[e + 2]), __uint_as_float(bb[e + 3])),
              pack_bf16x2(__uint_as_float(bb[e + 4]), __uint_as_float(bb[e + 5])),
              pack_bf16x2(__uint_as_float(bb[e + 6]), __uint_as_float(bb[e + 7])));
        }
      }
    } else if (ok && n_it == 0 && key < S) {
      // no query sees this key tile: its gradients are zero
      __nv_bfloat16* dk = args.dqkv + (int64_t)(row0 + key) * args.ld_dqkv + (args.Hq + g) * DH;
      __nv_bfloat16* dvp = args.dqkv + (int64_t)(row0 + key) * args.ld_dqkv + (args.Hq + args.Hkv + g) * DH;
      for (int e = wg * 8; e < DH; e += 8 * NG) {
        *reinterpret_cast<uint4*>(dk + e) = make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(dvp + e) = make_uint4(0, 0, 0, 0);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// D[b, h, q] = scale * sum_d dO[q, h, d] * O[q, h, d]  and  L2 = LSE * log2(e):
// both pre-scaled so the softmax backward spends one FFMA per element on each
// instead of a multiply and a subtract.  DH/8 lanes per (row, head), 16-byte
// loads; the same lanes zero the (row, head)'s fp32 dQ accumulator, which the
// main kernel reduce-adds into.
template <int DH>
__global__ void __launch_bounds__(256) attn_bwd_dot_kernel(const __nv_bfloat16* __restrict__ o, int64_t ldo,
                                                           const __nv_bfloat16* __restrict__ dout, int64_t lddo,
                                                           float* __restrict__ Dvec, const float* __restrict__ lse,
                                                           float* __restrict__ l2, float scale, int B, int S, int Hq,
                                                           float* __restrict__ dq_acc) {
  constexpr int LPR = DH / 8;  // lanes per (row, head)
  const int64_t gt = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t w = gt / LPR;  // (row, head) index
  const int sub = (int)(gt % LPR);
  const int64_t total = (int64_t)B * S * Hq;
  const bool ok = w < total;
  const int h = ok ? (int)(w % Hq) : 0;
  const int64_t row = ok ? w / Hq : 0;  // b*S + s
  float s = 0.f;
  if (ok) {
    const uint4 a = *reinterpret_cast<const uint4*>(o + row * ldo + h * DH + sub * 8);
    const uint4 c = *reinterpret_cast<const uint4*>(dout + row * lddo + h * DH + sub * 8);
    const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, cw[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 x = unpack_bf16x2(aw[e]), y = unpack_bf16x2(cw[e]);
      s += x.x * y.x + x.y * y.y;
    }
    float4* dqr = reinterpret_cast<float4*>(dq_acc + row * (int64_t)Hq * DH + h * DH + sub * 8);
    dqr[0] = make_float4(0.f, 0.f, 0.f, 0.f);
    dqr[1] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
#pragma unroll
  for (int off = LPR / 2; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  if (ok && sub == 0) {
    const int bb = (int)(row / S), q = (int)(row % S);
    const int64_t idx = ((int64_t)bb * Hq + h) * S + q;
    Dvec[idx] = s * scale;
    l2[idx] = lse[idx] * 1.4426950408889634f;
  }
}

__global__ void dq_convert_kernel(const float* __restrict__ acc, int64_t T, int ncols,
                                  __nv_bfloat16* __restrict__ dqkv, int64_t ld) {
  const int64_t n4 = T * ncols / 4;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < n4;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = idx * 4;
    const int64_t row = e / ncols;
    const int col = (int)(e % ncols);
    const float4 v = *reinterpret_cast<const float4*>(acc + e);
    *reinterpret_cast<uint2*>(dqkv + row * ld + col) = make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
  }
}

template <int DH>
static int launch_bwd(const LkAttnBwdDesc& d, cudaStream_t s) {
  using C = BwdCfg<DH>;
  const int64_t T = (int64_t)d.B * d.S;
  const int ncols = (d.Hq + 2 * d.Hkv) * DH;
  // dvec holds scale * D in its first half and LSE * log2(e) in the second
  float* l2 = d.dvec + lk_attn_dvec_half(d.B, d.Hq, d.S);
  // D = rowsum(dO * O)
  {
    const int64_t threads = T * d.Hq * (DH / 8);
    attn_bwd_dot_kernel<DH><<<(unsigned)cdiv(threads, 256), 256, 0, s>>>(
        (const __nv_bfloat16*)d.o, d.ld_o, (const __nv_bfloat16*)d.dout, d.ld_do, d.dvec, d.lse, l2, d.scale,
        d.B, d.S, d.Hq, d.dq_acc);
    if (check_launch("attn_bwd_dot")) return -1;
  }
  CUtensorMap tq, tdo, tdq;
  if (!make_tmap_2d(&tq, d.qkv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, T, ncols, d.ld_qkv, 128, 64)) return -1;
  if (!make_tmap_2d(&tdo, d.dout, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, T, (int64_t)d.Hq * DH, d.ld_do, 128, 64))
    return -1;
  // fp32 dQ accumulator [T, Hq*Dh]: 32 x 32 boxes (128-byte rows) for the bulk reduce-adds
  if (!make_tmap_2d(&tdq, d.dq_acc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, T, (int64_t)d.Hq * DH, (int64_t)d.Hq * DH,
                    32, 32))
    return -1;
  AttnBwdArgs a{};
  a.B = d.B;
  a.S = d.S;
  a.Hq = d.Hq;
  a.Hkv = d.Hkv;
  a.causal = d.causal;
  a.window = d.window;
  a.scale = d.scale;
  a.sl2 = d.scale * 1.4426950408889634f;
  a.lse = l2;
  a.Dvec = d.dvec;
  a.dq_acc = d.dq_acc;
  a.dqkv = (__nv_bfloat16*)d.dqkv;
  a.ld_dqkv = d.ld_dqkv;
  a.status = d.status;
  a.n_tiles = cdiv(d.S, 128);
  auto k = attn_bwd_kernel<DH>;
  cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  k<<<a.n_tiles * d.Hkv * d.B, 64 + 32 * bwd_softmax_warps<DH>(), C::SMEM, s>>>(tq, tdo, tdq, a);
  if (check_launch("attn_bwd")) return -1;
  const int64_t n4 = T * d.Hq * DH / 4;
  int grid_c = (int)std::min<int64_t>((n4 + 255) / 256, (int64_t)num_sms() * 16);
  dq_convert_kernel<<<grid_c, 256, 0, s>>>(d.dq_acc, T, d.Hq * DH, (__nv_bfloat16*)d.dqkv, d.ld_dqkv);
  return check_launch("attn_dq_convert");
}

}  // namespace lk

extern "C" int lk_attention_bwd(const LkAttnBwdDesc* d, cudaStream_t s) {
  using namespace lk;
  LK_REQUIRE(d->Hq % d->Hkv == 0, "attention_bwd: Hq must be a multiple of Hkv");
  LK_REQUIRE(d->ld_qkv % 8 == 0 && d->ld_do % 8 == 0 && d->ld_dqkv % 8 == 0 && d->ld_o % 8 == 0,
             "attention_bwd: row pitches must be multiples of 8");
  if (d->B == 0 || d->S == 0) return 0;
  if (d->Dh == 64) return launch_bwd<64>(*d, s);
  if (d->Dh == 128) return launch_bwd<128>(*d, s);
  return fail("attention_bwd: head_dim must be 64 or 128");
}
