// K3: causal / full flash-attention forward on tcgen05 (GQA, head_dim 64/128).
//
// Input is the packed QKV activation [B*S, (Hq + 2*Hkv) * Dh] produced by the
// QKV GEMM (+RoPE): query head h at column h*Dh, key head g at (Hq+g)*Dh and
// value head g at (Hq+Hkv+g)*Dh; q head h reads kv head h / (Hq/Hkv).
// Output O [B*S, Hq*Dh] bf16 and the natural-log LSE [B, Hq, S] fp32.
//
// One CTA per (128-query tile, q head, batch), 6 warps:
//   warp 0      TMA: Q once, then K_j / V_j into 2-stage rings (no multicast);
//   warp 1      one thread issues S = Q K_j^T (M=128, N=128) into TMEM and,
//               once P_j is in shared memory, O_j = P_j V_j (N = Dh) into a
//               second TMEM region;
//   warps 2..5  softmax: thread t of warp w owns query row 32*(w%4)+t, i.e.
//               TMEM lane; reads its S row, keeps the running max / sum in
//               registers, writes P (bf16, 128B-swizzled K-major) to shared
//               memory and accumulates O_j into a register accumulator with
//               the deferred rescale (acc = acc*alpha + O_j).
// The S of tile j+1 is computed while the softmax warps consume tile j.
//
// Replaces the reference's CPU attention: MultiHeadAttention::forward
// (src/nn/transformer_blocks.cpp:50-97), FlashAttentionV2::forward
// (include/nn/flash_attention.hpp:10-96, whose running-sum bug at :86 is not
// reproduced) and GroupedQueryAttention (include/nn/attention_variants.hpp:59).
#include "common.cuh"
#include "host_util.h"
#include "lk_api.h"

namespace lk {

struct AttnFwdArgs {
  int B, S, Hq, Hkv;  // S = query length
  int Skv;            // key length (== S for self-attention over packed QKV)
  int q_off;          // position of query 0 relative to key 0 (cached prefix length)
  int kcol0, vcol0;   // first column of key head 0 / value head 0 in the KV map
  int causal;
  int window;      // > 0: sliding window (keys in (q - window, q])
  float sl2;       // softmax scale * log2(e)
  __nv_bfloat16* o;
  int64_t ldo;
  float* lse;      // [B, Hq, S]
  int* status;
  int n_qtiles;
};

// 16-byte unit `u` (0..15, 8 bf16 each) of row `r` in a K-major 128B-swizzled
// [128 rows x 128 cols] bf16 tile stored as two [128 x 64] chunks.
__device__ __forceinline__ uint32_t sw128_off(int r, int u) {
  return (uint32_t)((u >> 3) * 16384 + r * 128 + (((u & 7) ^ (r & 7)) << 4));
}

template <int DH>
struct FwdCfg {
  static constexpr int QB = 128 * DH * 2;  // bytes of a [128 x DH] bf16 tile
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = QB;
  static constexpr int OFF_V = 3 * QB;
  static constexpr int OFF_P = 5 * QB;
  static constexpr int OFF_BAR = OFF_P + 32768;
  static constexpr int SMEM = OFF_BAR + 256;
  static constexpr int TMEM_COLS = 256;  // S: [0,128), O_j: [128, 128+DH)
  static constexpr int MIN_BLOCKS = DH == 64 ? 2 : 1;
};

template <int DH>
__global__ void __launch_bounds__(192, FwdCfg<DH>::MIN_BLOCKS)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tm_qkv, const __grid_constant__ CUtensorMap tm_kv,
                    const AttnFwdArgs args) {
  using C = FwdCfg<DH>;
  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t sbase = smem_u32(smem);
  if (sbase & 1023) {  // 128B-swizzled tiles need 1024-byte alignment
    if (threadIdx.x == 0) atomicCAS(args.status, 0, LK_ERR_BAD_INDEX);
    return;
  }
  const uint32_t bar = sbase + C::OFF_BAR;
  const uint32_t q_full = bar, k_full = bar + 8, k_empty = bar + 24, v_full = bar + 40,
                 v_empty = bar + 56, s_full = bar + 72, s_free = bar + 80, p_full = bar + 88,
                 o_full = bar + 96, drain = bar + 112;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_BAR + 128);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_BAR + 132);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // 1-D grid, heaviest causal q tiles first across all (head, batch) pairs
  const int hb = args.Hq * args.B;
  const int qt = args.n_qtiles - 1 - (int)(blockIdx.x / hb);
  const int h = (int)(blockIdx.x % hb) % args.Hq, b = (int)(blockIdx.x % hb) / args.Hq;
  const int kvh = h / (args.Hq / args.Hkv);
  const int S = args.S, Skv = args.Skv, q_off = args.q_off;
  const int nkv_all = (Skv + 127) / 128;
  const int qpos_max = q_off + qt * 128 + 127;  // largest query position in the tile
  int j_end = args.causal ? min(qpos_max / 128 + 1, nkv_all) : nkv_all;
  int j_begin = 0;
  if (args.window > 0) j_begin = max(0, (q_off + qt * 128 - args.window + 1) / 128);
  const int nkv = j_end - j_begin;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(k_full + 8 * s, 1);
      mbar_init(k_empty + 8 * s, 1);
      mbar_init(v_full + 8 * s, 1);
      mbar_init(v_empty + 8 * s, 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_free, 4);
    mbar_init(p_full, 4);
    mbar_init(o_full, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tm_qkv);
    tma_prefetch_desc(&tm_kv);
  }
  if (warp == 1) tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem, tO = tmem + 128;
  const int row0 = b * S;      // query rows
  const int krow0 = b * Skv;   // key / value rows

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ TMA
      uint32_t pending = 0, parbits = 0;  // bit0..1: K stages, bit2..3: V stages
      mbar_expect_tx(q_full, C::QB);
#pragma unroll
      for (int c = 0; c < DH / 64; ++c)
        tma_load_2d(sbase + C::OFF_Q + c * 16384, &tm_qkv, q_full, h * DH + c * 64,
                    row0 + qt * 128);
      bool ok = true;
      for (int jj = 0; jj < nkv && ok; ++jj) {
        const int j = j_begin + jj;
        const int st = jj & 1;
        const uint32_t ph = (jj >> 1) & 1;
        if (!bounded_wait(k_empty + 8 * st, ph ^ 1, args.status, LK_ERR_TIMEOUT_EMPTY, abort_flag)) {
          ok = false;
          break;
        }
        mbar_expect_tx(k_full + 8 * st, C::QB);
#pragma unroll
        for (int c = 0; c < DH / 64; ++c)
          tma_load_2d(sbase + C::OFF_K + st * C::QB + c * 16384, &tm_kv, k_full + 8 * st,
                      args.kcol0 + kvh * DH + c * 64, krow0 + j * 128);
        pending |= 1u << st;
        parbits = (parbits & ~(1u << st)) | (ph << st);
        if (!bounded_wait(v_empty + 8 * st, ph ^ 1, args.status, LK_ERR_TIMEOUT_EMPTY, abort_flag)) {
          ok = false;
          break;
        }
        mbar_expect_tx(v_full + 8 * st, C::QB);
#pragma unroll
        for (int c = 0; c < DH / 64; ++c)
          tma_load_2d(sbase + C::OFF_V + st * C::QB + c * 16384, &tm_kv, v_full + 8 * st,
                      args.vcol0 + kvh * DH + c * 64, krow0 + j * 128);
        pending |= 4u << st;
        parbits = (parbits & ~(4u << st)) | (ph << (st + 2));
      }
      if (!ok) {
        bounded_wait(q_full, 0, args.status, LK_ERR_TIMEOUT_DRAIN, nullptr);
        for (int i = 0; i < 2; ++i) {
          if (pending & (1u << i))
            bounded_wait(k_full + 8 * i, (parbits >> i) & 1, args.status, LK_ERR_TIMEOUT_DRAIN, nullptr);
          if (pending & (4u << i))
            bounded_wait(v_full + 8 * i, (parbits >> (i + 2)) & 1, args.status, LK_ERR_TIMEOUT_DRAIN, nullptr);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------ MMA
      constexpr uint32_t idesc_s = make_idesc_bf16(128, 128, false, false);
      constexpr uint32_t idesc_o = make_idesc_bf16(128, DH, false, true);
      const uint32_t sq = sbase + C::OFF_Q, sp = sbase + C::OFF_P;
      bool ok = bounded_wait(q_full, 0, args.status, LK_ERR_TIMEOUT_FULL, abort_flag);
      auto issue_s = [&](int jj) -> bool {
        const int st = jj & 1;
        if (!bounded_wait(k_full + 8 * st, (jj >> 1) & 1, args.status, LK_ERR_TIMEOUT_FULL, abort_flag))
          return false;
        if (jj > 0 && !bounded_wait(s_free, (jj - 1) & 1, args.status, LK_ERR_TIMEOUT_ACCUM, abort_flag))
          return false;
        tc_fence_after();
        const uint32_t sk = sbase + C::OFF_K + st * C::QB;
#pragma unroll
        for (int kk = 0; kk < DH / 16; ++kk) {
          const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
          tc_mma_f16(tS, make_desc_sw128(sq + off, 16, 1024), make_desc_sw128(sk + off, 16, 1024),
                     idesc_s, kk > 0 ? 1u : 0u);
        }
        tc_commit(s_full);
        tc_commit(k_empty + 8 * st);
        return true;
      };
      if (ok && nkv > 0) ok = issue_s(0);
      for (int jj = 0; jj < nkv && ok; ++jj) {
        if (jj + 1 < nkv && !issue_s(jj + 1)) {
          ok = false;
          break;
        }
        const int st = jj & 1;
        if (!bounded_wait(p_full, jj & 1, args.status, LK_ERR_TIMEOUT_ACCUM, abort_flag) ||
            !bounded_wait(v_full + 8 * st, (jj >> 1) & 1, args.status, LK_ERR_TIMEOUT_FULL, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sv = sbase + C::OFF_V + st * C::QB;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {  // 128 keys, 16 per MMA
          const uint64_t ad = make_desc_sw128(sp + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = make_desc_sw128(sv + kk * 2048, 16384, 1024);
          tc_mma_f16(tO, ad, bd, idesc_o, (jj > 0 || kk > 0) ? 1u : 0u);
        }
        tc_commit(o_full);
        tc_commit(v_empty + 8 * st);
      }
      tc_commit(drain);
      bounded_wait(drain, 0, args.status, LK_ERR_TIMEOUT_DRAIN, nullptr);
    }
  } else {
    // ---------------------------------------------------------- softmax
    // O accumulates in TMEM across key tiles.  Each row keeps the max m_used
    // its exponentials are taken against and rescales its O row (TMEM
    // read-modify-write) only when a tile's max exceeds m_used by more than 8
    // (a factor 256), so P stays <= 256 and most tiles need no O traffic.
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // query row within the tile
    const int ql = qt * 128 + r;        // query row within the sequence
    const int q = q_off + ql;           // query position (keys are 0..Skv-1)
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    uint8_t* sP = smem + C::OFF_P;
    float m_used = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int jj = 0; jj < nkv; ++jj) {
      const int j = j_begin + jj;
      bool w_ok = bounded_wait(s_full, jj & 1, args.status, LK_ERR_TIMEOUT_ACCUM, abort_flag);
      if (!__all_sync(0xffffffffu, w_ok)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sv[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(tS + lane_off + c * 32, sv[c]);
      tc_wait_ld();
      // S is in registers: release the TMEM buffer so S_{j+1} can start now
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(s_free);
      const bool need_mask = (args.causal && j * 128 + 127 > q_off + qt * 128) || (j + 1) * 128 > Skv ||
                             (args.window > 0 && j * 128 <= q - args.window + 127);
      float mraw = -INFINITY;  // max of the raw scores (scale > 0 commutes with max)
      if (need_mask) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const int key = j * 128 + c * 32 + e;
            if (key >= Skv || (args.causal && key > q) || (args.window > 0 && key <= q - args.window))
              sv[c][e] = __float_as_uint(-INFINITY);
          }
        }
      }
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int e = 0; e < 32; ++e) mraw = fmaxf(mraw, __uint_as_float(sv[c][e]));
      const float mx = mraw * args.sl2;
      const float m_new = (mx > m_used + 8.f) ? mx : m_used;
      const float alpha = (m_new != m_used) ? fast_exp2(m_used - m_new) : 1.f;
      const float mb = (m_new == -INFINITY) ? 0.f : m_new;
      // P packed to bf16 pairs in place: sv[c][0..15] hold chunk c's 32 probabilities
      float rowsum = 0.f;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          const float p0 = fast_exp2(fmaf(__uint_as_float(sv[c][e]), args.sl2, -mb));
          const float p1 = fast_exp2(fmaf(__uint_as_float(sv[c][e + 1]), args.sl2, -mb));
          rowsum += p0 + p1;
          sv[c][e >> 1] = pack_bf16x2(p0, p1);
        }
      }
      // PV_{j-1} must be done before O is rescaled and before P is overwritten
      if (jj > 0) {
        w_ok = bounded_wait(o_full, (jj - 1) & 1, args.status, LK_ERR_TIMEOUT_ACCUM, abort_flag);
        if (!__all_sync(0xffffffffu, w_ok)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll 1
          for (int c = 0; c < DH / 32; ++c) {
            uint32_t ov[32];
            tmem_ld32(tO + lane_off + c * 32, ov);
            tc_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) ov[e] = __float_as_uint(__uint_as_float(ov[e]) * alpha);
            tmem_st32(tO + lane_off + c * 32, ov);
          }
          tc_wait_st();
        }
      }
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        const uint32_t* pk = &sv[u >> 2][(u & 3) * 4];
        *reinterpret_cast<uint4*>(sP + sw128_off(r, u)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      }
      tc_fence_before();
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
      l_run = l_run * alpha + rowsum;
      m_used = m_new;
    }
    if (ok && nkv > 0) {
      bool w_ok = bounded_wait(o_full, (nkv - 1) & 1, args.status, LK_ERR_TIMEOUT_ACCUM, abort_flag);
      if (__all_sync(0xffffffffu, w_ok)) {
        tc_fence_after();
        const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
        __nv_bfloat16* orow = args.o + (int64_t)(row0 + ql) * args.ldo + h * DH;
#pragma unroll 1
        for (int c = 0; c < DH / 32; ++c) {
          uint32_t v[32];
          tmem_ld32(tO + lane_off + c * 32, v);
          tc_wait_ld();
          if (ql < S) {
#pragma unroll
            for (int d = 0; d < 32; d += 8)
              *reinterpret_cast<uint4*>(orow + c * 32 + d) = make_uint4(
                  pack_bf16x2(__uint_as_float(v[d]) * inv, __uint_as_float(v[d + 1]) * inv),
                  pack_bf16x2(__uint_as_float(v[d + 2]) * inv, __uint_as_float(v[d + 3]) * inv),
                  pack_bf16x2(__uint_as_float(v[d + 4]) * inv, __uint_as_float(v[d + 5]) * inv),
                  pack_bf16x2(__uint_as_float(v[d + 6]) * inv, __uint_as_float(v[d + 7]) * inv));
          }
        }
        // natural-log LSE: (m + log2 l) * ln 2
        if (ql < S)
          args.lse[((int64_t)b * args.Hq + h) * S + ql] =
              l_run > 0.f ? (m_used + log2f(l_run)) * 0.69314718055994531f : -INFINITY;
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

template <int DH>
static int launch_fwd(const LkAttnDesc& d, cudaStream_t s) {
  using C = FwdCfg<DH>;
  const bool packed = d.kv == nullptr;
  const int Skv = packed ? d.S : d.Skv;
  const int64_t qcols = packed ? (int64_t)(d.Hq + 2 * d.Hkv) * DH : (int64_t)d.Hq * DH;
  CUtensorMap tm, tkv;
  if (!make_tmap_2d(&tm, d.qkv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (int64_t)d.B * d.S, qcols,
                    d.ld_qkv, 128, 64))
    return -1;
  if (packed) {
    tkv = tm;
  } else if (!make_tmap_2d(&tkv, d.kv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (int64_t)d.B * Skv,
                           (int64_t)2 * d.Hkv * DH, d.ld_kv, 128, 64)) {
    return -1;
  }
  AttnFwdArgs a{};
  a.B = d.B;
  a.S = d.S;
  a.Skv = Skv;
  a.q_off = packed ? 0 : d.q_off;
  a.kcol0 = packed ? d.Hq * DH : 0;
  a.vcol0 = packed ? (d.Hq + d.Hkv) * DH : d.Hkv * DH;
  a.Hq = d.Hq;
  a.Hkv = d.Hkv;
  a.causal = d.causal;
  a.window = d.window;
  a.sl2 = d.scale * 1.4426950408889634f;
  a.o = (__nv_bfloat16*)d.o;
  a.ldo = d.ld_o;
  a.lse = d.lse;
  a.status = d.status;
  a.n_qtiles = cdiv(d.S, 128);
  auto k = attn_fwd_kernel<DH>;
  cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  k<<<a.n_qtiles * d.Hq * d.B, 192, C::SMEM, s>>>(tm, tkv, a);
  return check_launch("attn_fwd");
}

}  // namespace lk

extern "C" int lk_attention_fwd(const LkAttnDesc* d, cudaStream_t s) {
  using namespace lk;
  LK_REQUIRE(d->Hq % d->Hkv == 0, "attention: Hq must be a multiple of Hkv");
  LK_REQUIRE(d->ld_qkv % 8 == 0 && d->ld_o % 8 == 0, "attention: row pitches must be multiples of 8");
  if (d->B == 0 || d->S == 0) return 0;
  if (d->Dh == 64) return launch_fwd<64>(*d, s);
  if (d->Dh == 128) return launch_fwd<128>(*d, s);
  return fail("attention: head_dim must be 64 or 128");
}
