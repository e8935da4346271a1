// K3: causal / full flash-attention forward on tcgen05 (GQA, head_dim 64/128).
//
// Input is the packed QKV activation [B*S, (Hq + 2*Hkv) * Dh] produced by the
// QKV GEMM (+RoPE): query head h at column h*Dh, key head g at (Hq+g)*Dh and
// value head g at (Hq+Hkv+g)*Dh; q head h reads kv head h / (Hq/Hkv).
// Output O [B*S, Hq*Dh] bf16 and the natural-log LSE [B, Hq, S] fp32.
//
// One CTA per (pair of 128-query tiles a/b, q head, batch), 10 warps:
//   warp 0      TMA: both Q tiles once, then K_j / V_j into 2-3 stage rings
//               shared by the two tiles (no multicast);
//   warp 1      one thread issues S_t = Q_t K_j^T (M=128, N=128) into TMEM and,
//               once P_t is back in TMEM, O_t += P_t V_j with P_t as the
//               tensor-memory A operand; the tensor cores serve one softmax
//               group while the other works (ping-pong).  Head dim 128: order
//               PV_a(j), S_a(j+1), PV_b(j), S_b(j+1), P over S.  Head dim 64: P
//               has its own columns, so S_t(j+1) goes out as soon as group t has
//               read S_t(j), ahead of the PVs;
//   warps 2..9  two softmax groups of 4 warps (tile a, tile b): thread = query
//               row = TMEM lane; it reads its 128 scores, keeps the running
//               max / sum in registers, writes P as bf16 pairs and rescales its
//               O row in TMEM only when the max grew by more than 2^8.
// Replaces the reference's CPU attention: MultiHeadAttention::forward
// (src/nn/transformer_blocks.cpp:50-97), FlashAttentionV2::forward
// (include/nn/flash_attention.hpp:10-96, whose running-sum bug at :86 is not
// reproduced) and GroupedQueryAttention (include/nn/attention_variants.hpp:59).
#include <cstdlib>

#include "common.cuh"
#include "host_util.h"
#include "lk_api.h"

namespace lk {

// 2^x on the FMA pipe (offloads the MUFU, which bounds the head_dim-64
// softmax): round-to-nearest range reduction x = n + f, f in [-1/2, 1/2], by
// adding 1.5 * 2^23; p(f) a cubic fitted here by iteratively reweighted least
// squares to minimise the relative error of 2^f (max 9.1e-5 in fp32, far
// below bf16's 2^-9 rounding of P); 2^n by adding n to the exponent bits.
// Valid for x >= -126 (the caller clamps) and x < 128.
__device__ __forceinline__ float exp2_fma(float x) {
  x = fmaxf(x, -126.f);
  const float t = x + 12582912.f;
  const float n = t - 12582912.f;
  const float f = x - n;
  float p = fmaf(f, 0.055171433836221695f, 0.24261081218719482f);
  p = fmaf(f, p, 0.6932609677314758f);
  p = fmaf(f, p, 0.9999281167984009f);
  return __uint_as_float(__float_as_uint(p) + (__float_as_uint(t) << 23));
}

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
  int n_qtiles;  // CTAs per (head, batch): pairs of 128-query tiles
  int emu;       // exponentials per 16 computed on the FMA pipe (0, 2 or 4)
};

template <int DH>
struct FwdCfg {
  static constexpr int QB = 128 * DH * 2;  // bytes of a [128 x DH] bf16 tile
  static constexpr int NS = DH == 64 ? 3 : 2;  // K / V stages
  static constexpr int OFF_Q = 0;              // two query tiles
  static constexpr int OFF_K = 2 * QB;
  static constexpr int OFF_V = OFF_K + NS * QB;
  static constexpr int OFF_BAR = OFF_V + NS * QB;
  static constexpr int OFF_XCH = OFF_BAR + 256;  // split softmax: row-max exchange slots (4 KB)
  static constexpr int SMEM = OFF_XCH + 4096;
  static constexpr int TMEM_COLS = 512;  // S_a, S_b, O_a, O_b (+ P_a, P_b at head dim 64)
  // TMA warp, MMA warp, two groups of 4 softmax warps (thread = query row) or,
  // with split rows, two groups of 8 (two threads per row, 64 keys each)
  static constexpr int threads(int split) { return 64 + 32 * 4 * split * 2; }
};

template <int DH, int EMU, int SPLIT>
__global__ void __launch_bounds__(FwdCfg<DH>::threads(SPLIT), 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tm_qkv, const __grid_constant__ CUtensorMap tm_kv,
                    const AttnFwdArgs args) {
  using C = FwdCfg<DH>;
  constexpr int NS = C::NS;
  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t sbase = smem_u32(smem);
  if (sbase & 1023) {  // 128B-swizzled tiles need 1024-byte alignment
    if (threadIdx.x == 0) atomicCAS(args.status, 0, LK_ERR_BAD_INDEX);
    return;
  }
  const uint32_t bar = sbase + C::OFF_BAR;
  // [0] q_full, [1..3] k_full, [4..6] k_empty, [7..9] v_full, [10..12] v_empty,
  // [13,14] s_full[t], [15,16] p_full[t], [17,18] o_done[t], [19] drain, [20,21] s_free[t]
  const uint32_t q_full = bar, k_full = bar + 8, k_empty = bar + 32, v_full = bar + 56, v_empty = bar + 80,
                 s_full = bar + 104, p_full = bar + 120, o_done = bar + 136, drain = bar + 152,
                 s_free = bar + 160;
  // Head dim 64 (one thread per row): P gets its own TMEM columns instead of
  // overwriting S, so S(j+1) is computed while the softmax still turns S(j) into
  // P(j): TMEM = S_a, S_b (128 each) | P_a, P_b (64) | O_a, O_b (64).  Otherwise
  // P is written over S: S_a, S_b | O_a, O_b (DH each).
  constexpr bool SEP = DH == 64 && SPLIT == 1;
  constexpr uint32_t P_COL = SEP ? 256 : 0, O_COL = SEP ? 384 : 256;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_BAR + 192);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_BAR + 196);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // 1-D grid, heaviest causal query pairs first across all (head, batch) pairs
  const int hb = args.Hq * args.B;
  const int qp = args.n_qtiles - 1 - (int)(blockIdx.x / hb);  // n_qtiles counts 256-query pairs here
  const int h = (int)(blockIdx.x % hb) % args.Hq, b = (int)(blockIdx.x % hb) / args.Hq;
  const int kvh = h / (args.Hq / args.Hkv);
  const int S = args.S, Skv = args.Skv, q_off = args.q_off;
  const int nkv_all = (Skv + 127) / 128;
  // key-tile range [jb[t], je[t]) of query tile t (qt = 2 qp + t); empty past the sequence
  auto key_range = [&](int qt, int& lo, int& hi) {
    lo = hi = 0;
    if (qt * 128 >= S) return;
    const int qpos_max = q_off + qt * 128 + 127;
    hi = args.causal ? min(qpos_max / 128 + 1, nkv_all) : nkv_all;
    lo = args.window > 0 ? max(0, (q_off + qt * 128 - args.window + 1) / 128) : 0;
    if (hi < lo) hi = lo;
  };
  int jb0, je0, jb1, je1;
  key_range(2 * qp, jb0, je0);
  key_range(2 * qp + 1, jb1, je1);
  const int j_lo = je0 > jb0 ? jb0 : jb1;
  const int j_hi = max(je0, je1);
  const int nkv = max(0, j_hi - j_lo);  // key tiles loaded (union of both ranges)
  auto active = [&](int t, int j) { return t == 0 ? (j >= jb0 && j < je0) : (j >= jb1 && j < je1); };

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s2 = 0; s2 < NS; ++s2) {
      mbar_init(k_full + 8 * s2, 1);
      mbar_init(k_empty + 8 * s2, 1);
      mbar_init(v_full + 8 * s2, 1);
      mbar_init(v_empty + 8 * s2, 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(s_full + 8 * t, 1);
      mbar_init(p_full + 8 * t, 4 * SPLIT);
      mbar_init(o_done + 8 * t, 1);
      mbar_init(s_free + 8 * t, 4 * SPLIT);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tm_qkv);
    tma_prefetch_desc(&tm_kv);
  }
  if (SPLIT == 2)
    for (int i = threadIdx.x; i < 512; i += blockDim.x)
      reinterpret_cast<unsigned long long*>(smem + C::OFF_XCH)[i] = 0ull;  // sequence 0: never used
  if (warp == 1) tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int row0 = b * S;      // query rows
  const int krow0 = b * Skv;   // key / value rows

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ TMA
      uint32_t pending = 0, parbits = 0;  // bits 0..NS-1: K stages, NS..2NS-1: V stages
      mbar_expect_tx(q_full, 2 * C::QB);
#pragma unroll
      for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int c = 0; c < DH / 64; ++c)
          tma_load_2d(sbase + C::OFF_Q + t * C::QB + c * 16384, &tm_qkv, q_full, h * DH + c * 64,
                      row0 + (2 * qp + t) * 128);
      bool ok = true;
      for (int u = 0; u < nkv && ok; ++u) {
        const int j = j_lo + u;
        const int st = u % NS;
        const uint32_t ph = (uint32_t)(u / NS) & 1;
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
        pending |= 1u << (NS + st);
        parbits = (parbits & ~(1u << (NS + st))) | (ph << (NS + st));
      }
      if (!ok) {
        bounded_wait(q_full, 0, args.status, LK_ERR_TIMEOUT_DRAIN, nullptr);
        for (int i = 0; i < NS; ++i) {
          if (pending & (1u << i))
            bounded_wait(k_full + 8 * i, (parbits >> i) & 1, args.status, LK_ERR_TIMEOUT_DRAIN, nullptr);
          if (pending & (1u << (NS + i)))
            bounded_wait(v_full + 8 * i, (parbits >> (NS + i)) & 1, args.status, LK_ERR_TIMEOUT_DRAIN, nullptr);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------ MMA
      // Ping-pong: PV_a(j), S_a(j+1), PV_b(j), S_b(j+1): while one softmax group
      // works on its tile the tensor cores serve the other.  MMAs of one thread
      // run in issue order, so S_t(j+1) overwriting P_t(j) in TMEM follows PV_t(j).
      constexpr uint32_t idesc_s = make_idesc_bf16(128, 128, false, false);
      constexpr uint32_t idesc_o = make_idesc_bf16(128, DH, false, true);
      bool ok = bounded_wait(q_full, 0, args.status, LK_ERR_TIMEOUT_FULL, abort_flag);
      int n_pv0 = 0, n_pv1 = 0;  // PV MMAs issued per tile (= their p_full phase counters)
      auto issue_s = [&](int t, int u) {
        const int st = u % NS;
        const uint32_t sq = sbase + C::OFF_Q + t * C::QB, sk = sbase + C::OFF_K + st * C::QB;
        const uint32_t tS = tmem + 128 * t;
#pragma unroll
        for (int kk = 0; kk < DH / 16; ++kk) {
          const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
          tc_mma_f16(tS, make_desc_sw128(sq + off, 16, 1024), make_desc_sw128(sk + off, 16, 1024), idesc_s,
                     kk > 0 ? 1u : 0u);
        }
        tc_commit(s_full + 8 * t);
      };
      auto issue_pv = [&](int t, int u) -> bool {
        int& npv = t == 0 ? n_pv0 : n_pv1;
        if (!bounded_wait(p_full + 8 * t, npv & 1, args.status, LK_ERR_TIMEOUT_ACCUM, abort_flag)) return false;
        tc_fence_after();
        const int st = u % NS;
        const uint32_t sv = sbase + C::OFF_V + st * C::QB;
        const uint32_t tP = SEP ? tmem + P_COL + 64 * t : tmem + 128 * t, tO = tmem + O_COL + DH * t;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)  // 128 keys, 16 per MMA; P (bf16 pairs) from TMEM
          tc_mma_f16_ta(tO, tP + kk * 8, make_desc_sw128(sv + kk * 2048, 16384, 1024), idesc_o,
                        (npv > 0 || kk > 0) ? 1u : 0u);
        tc_commit(o_done + 8 * t);
        ++npv;
        return true;
      };
      if (ok && nkv > 0) {
        ok = bounded_wait(k_full, 0, args.status, LK_ERR_TIMEOUT_FULL, abort_flag);
        if (ok) {
          tc_fence_after();
          for (int t = 0; t < 2; ++t)
            if (active(t, j_lo)) issue_s(t, 0);
          tc_commit(k_empty);
        }
      }
      int n_s[2] = {active(0, j_lo) ? 1 : 0, active(1, j_lo) ? 1 : 0};  // S MMAs issued per tile
      for (int u = 0; u < nkv && ok && SEP; ++u) {
        // S_t(j+1) once the softmax of tile t has read S_t(j) (s_free), then the PVs
        const int j = j_lo + u;
        const int st = u % NS;
        const bool nxt = u + 1 < nkv;
        const int st1 = (u + 1) % NS;
        if (nxt) {
          if (!bounded_wait(k_full + 8 * st1, ((u + 1) / NS) & 1, args.status, LK_ERR_TIMEOUT_FULL, abort_flag)) {
            ok = false;
            break;
          }
          for (int t = 0; t < 2 && ok; ++t) {
            if (!active(t, j + 1)) continue;
            if (n_s[t] > 0)
              ok = bounded_wait(s_free + 8 * t, (n_s[t] - 1) & 1, args.status, LK_ERR_TIMEOUT_ACCUM, abort_flag);
            if (!ok) break;
            tc_fence_after();
            issue_s(t, u + 1);
            ++n_s[t];
          }
          if (!ok) break;
          tc_commit(k_empty + 8 * st1);
        }
        if (!bounded_wait(v_full + 8 * st, (u / NS) & 1, args.status, LK_ERR_TIMEOUT_FULL, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if ((active(0, j) && !issue_pv(0, u)) || (active(1, j) && !issue_pv(1, u))) {
          ok = false;
          break;
        }
        tc_commit(v_empty + 8 * st);
      }
      for (int u = 0; u < nkv && ok && !SEP; ++u) {
        const int j = j_lo + u;
        const int st = u % NS;
        const bool nxt = u + 1 < nkv;
        const int st1 = (u + 1) % NS;
        if (!bounded_wait(v_full + 8 * st, (u / NS) & 1, args.status, LK_ERR_TIMEOUT_FULL, abort_flag)) {
          ok = false;
          break;
        }
        if (nxt && !bounded_wait(k_full + 8 * st1, ((u + 1) / NS) & 1, args.status, LK_ERR_TIMEOUT_FULL,
                                 abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (active(0, j) && !issue_pv(0, u)) {
          ok = false;
          break;
        }
        if (nxt && active(0, j + 1)) issue_s(0, u + 1);
        if (active(1, j) && !issue_pv(1, u)) {
          ok = false;
          break;
        }
        tc_commit(v_empty + 8 * st);
        if (nxt && active(1, j + 1)) issue_s(1, u + 1);
        if (nxt) tc_commit(k_empty + 8 * st1);
      }
      tc_commit(drain);
      bounded_wait(drain, 0, args.status, LK_ERR_TIMEOUT_DRAIN, nullptr);
    }
  } else if constexpr (SPLIT == 2) {
    // ------------------------------------------------- softmax, split rows
    // Group t (warps 2..9: tile a, 10..17: tile b), 8 warps: two threads per
    // query row (the warps w and w + 4 share TMEM lane quarter w % 4), each
    // owning 64 of the tile's 128 keys, so each SMSP has two softmax warps per
    // group to hide TMEM and MUFU latency.  The partners exchange their row max
    // through a 64-bit {sequence, value} slot in shared memory (a bounded poll,
    // no named barrier); sums stay per half until the end.  A thread cannot
    // write its next slot before its partner read the last one: the next S
    // tile needs both halves' P of this one (p_full counts all 8 warps).
    const int t = (warp - 2) >> 3;
    const int hf = ((warp - 2) >> 2) & 1;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const int qt = 2 * qp + t;
    const int ql = qt * 128 + r;
    const int q = q_off + ql;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t tS = tmem + 128 * t + lane_off, tO = tmem + O_COL + DH * t + lane_off;
    const int jbt = t == 0 ? jb0 : jb1;
    const int n_t = (t == 0 ? je0 : je1) - jbt;
    volatile unsigned long long* xch = reinterpret_cast<volatile unsigned long long*>(smem + C::OFF_XCH);
    volatile unsigned long long* mine = xch + ((t * 4 + quarter) * 2 + hf) * 32 + lane;
    volatile unsigned long long* theirs = xch + ((t * 4 + quarter) * 2 + (hf ^ 1)) * 32 + lane;
    auto exchange = [&](uint32_t seq, float v, float& other) -> bool {
      *mine = ((unsigned long long)seq << 32) | __float_as_uint(v);
      const uint64_t t0 = globaltimer();
      while (true) {
        const unsigned long long x = *theirs;
        if ((uint32_t)(x >> 32) == seq) {
          other = __uint_as_float((uint32_t)x);
          return true;
        }
        if (*abort_flag) return false;
        if (globaltimer() - t0 > LK_WAIT_TIMEOUT_NS) {
          atomicCAS(args.status, 0, LK_ERR_TIMEOUT_ACCUM);
          *abort_flag = 1;
          return false;
        }
      }
    };
    float m_used = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int jj = 0; jj < n_t; ++jj) {
      const int j = jbt + jj;
      bool w_ok = bounded_wait(s_full + 8 * t, jj & 1, args.status, LK_ERR_TIMEOUT_ACCUM, abort_flag);
      if (!__all_sync(0xffffffffu, w_ok)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const bool need_mask = (args.causal && j * 128 + 127 > q_off + qt * 128) || (j + 1) * 128 > Skv ||
                             (args.window > 0 && j * 128 <= q - args.window + 127);
      const int kbase = j * 128 + 64 * hf;  // this thread's 64 keys
      const int khi = min(Skv - 1, args.causal ? q : Skv - 1) - kbase;
      const int klo = (args.window > 0 ? q - args.window + 1 : 0) - kbase;
      auto mask_chunk = [&](uint32_t (&x)[32], int c) {
        if (!need_mask) return;
#pragma unroll
        for (int e = 0; e < 32; ++e)
          if (c * 32 + e > khi || c * 32 + e < klo) x[e] = __float_as_uint(-INFINITY);
      };
      uint32_t s0[32], s1[32];
      tmem_ld32(tS + 64 * hf, s0);
      tmem_ld32(tS + 64 * hf + 32, s1);
      tc_wait_ld();
      mask_chunk(s0, 0);
      mask_chunk(s1, 1);
      float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int e = 0; e < 32; ++e)
        m4[e & 3] = fmaxf(m4[e & 3], fmaxf(__uint_as_float(s0[e]), __uint_as_float(s1[e])));
      float mother = -INFINITY;
      w_ok = exchange((uint32_t)jj + 1u, fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3])), mother);
      if (!__all_sync(0xffffffffu, w_ok)) {
        ok = false;
        break;
      }
      const float mraw = fmaxf(fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3])), mother);
      const float mx = mraw * args.sl2;
      const float m_new = (mx > m_used + 8.f) ? mx : m_used;
      const float alpha = (m_new != m_used) ? fast_exp2(m_used - m_new) : 1.f;
      const float mb = (m_new == -INFINITY) ? 0.f : m_new;
      // P as bf16 pairs: keys [64 hf + 32 c, +32) -> TMEM columns 32 hf + 16 c (the
      // partner's scores there are already in its registers: it exchanged its max)
      float r4[4] = {0.f, 0.f, 0.f, 0.f};
      auto emit = [&](const uint32_t (&x)[32], int c) {
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          const float p0 = fast_exp2(fmaf(__uint_as_float(x[e]), args.sl2, -mb));
          const float p1 = fast_exp2(fmaf(__uint_as_float(x[e + 1]), args.sl2, -mb));
          r4[(e >> 1) & 3] += p0 + p1;
          pk[e >> 1] = pack_bf16x2(p0, p1);
        }
        tmem_st16(tS + 32 * hf + 16 * c, pk);
      };
      emit(s0, 0);
      emit(s1, 1);
      const float rowsum = (r4[0] + r4[1]) + (r4[2] + r4[3]);
      // rescale this half of the O row (rare): PV(jj-1) must have finished
      if (jj > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
        w_ok = bounded_wait(o_done + 8 * t, (jj - 1) & 1, args.status, LK_ERR_TIMEOUT_ACCUM, abort_flag);
        if (!__all_sync(0xffffffffu, w_ok)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < DH / 64; ++c) {
          uint32_t ov[32];
          tmem_ld32(tO + hf * (DH / 2) + c * 32, ov);
          tc_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) ov[e] = __float_as_uint(__uint_as_float(ov[e]) * alpha);
          tmem_st32(tO + hf * (DH / 2) + c * 32, ov);
        }
      }
      tc_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full + 8 * t);
      l_run = l_run * alpha + rowsum;
      m_used = m_new;
    }
    if (ok && n_t > 0) {
      bool w_ok = bounded_wait(o_done + 8 * t, (n_t - 1) & 1, args.status, LK_ERR_TIMEOUT_ACCUM, abort_flag);
      float lother = 0.f;
      w_ok = w_ok && exchange(0x7FFFFFFFu, l_run, lother);
      if (__all_sync(0xffffffffu, w_ok)) {
        tc_fence_after();
        const float l_tot = l_run + lother;
        const float inv = l_tot > 0.f ? 1.f / l_tot : 0.f;
        __nv_bfloat16* orow = args.o + (int64_t)(row0 + ql) * args.ldo + h * DH + hf * (DH / 2);
#pragma unroll 1
        for (int c = 0; c < DH / 64; ++c) {
          uint32_t v[32];
          tmem_ld32(tO + hf * (DH / 2) + c * 32, v);
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
        if (ql < S && hf == 0)
          args.lse[((int64_t)b * args.Hq + h) * S + ql] =
              l_tot > 0.f ? (m_used + log2f(l_tot)) * 0.69314718055994531f : -INFINITY;
      }
    }
  } else {
    // ---------------------------------------------------------- softmax
    // Group t (warps 2..5: tile a, 6..9: tile b); thread = query row (TMEM lane).
    // O accumulates in TMEM across key tiles.  Each row keeps the max m_used
    // its exponentials are taken against and rescales its O row (TMEM
    // read-modify-write) only when a tile's max exceeds m_used by more than 8
    // (a factor 256), so P stays <= 256 and most tiles need no O traffic.
    const int t = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // query row within the tile
    const int qt = 2 * qp + t;
    const int ql = qt * 128 + r;        // query row within the sequence
    const int q = q_off + ql;           // query position (keys are 0..Skv-1)
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t tS = tmem + 128 * t + lane_off, tO = tmem + O_COL + DH * t + lane_off;
    const uint32_t tP = SEP ? tmem + P_COL + 64 * t + lane_off : tS;
    const int jbt = t == 0 ? jb0 : jb1;
    const int n_t = (t == 0 ? je0 : je1) - jbt;
    float m_used = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int jj = 0; jj < n_t; ++jj) {
      const int j = jbt + jj;
      bool w_ok = bounded_wait(s_full + 8 * t, jj & 1, args.status, LK_ERR_TIMEOUT_ACCUM, abort_flag);
      if (!__all_sync(0xffffffffu, w_ok)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const bool need_mask = (args.causal && j * 128 + 127 > q_off + qt * 128) || (j + 1) * 128 > Skv ||
                             (args.window > 0 && j * 128 <= q - args.window + 127);
      // keys of this tile the row may see: [klo, khi] relative to the tile start
      const int kbase = j * 128;
      const int khi = min(Skv - 1, args.causal ? q : Skv - 1) - kbase;
      const int klo = (args.window > 0 ? q - args.window + 1 : 0) - kbase;
      auto mask_chunk = [&](uint32_t (&x)[32], int c) {
        if (!need_mask) return;
#pragma unroll
        for (int e = 0; e < 32; ++e)
          if (c * 32 + e > khi || c * 32 + e < klo) x[e] = __float_as_uint(-INFINITY);
      };
      // pass 1: all 128 scores of the row in registers with one TMEM round trip,
      // then the row max (four independent max chains)
      uint32_t s0[32], s1[32], s2[32], s3[32];
      float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
      tmem_ld32(tS, s0);
      tmem_ld32(tS + 32, s1);
      tmem_ld32(tS + 64, s2);
      tmem_ld32(tS + 96, s3);
      tc_wait_ld();
      if constexpr (SEP) {
        // S is in registers: the MMA warp may compute the next S into these columns
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(s_free + 8 * t);
      }
      mask_chunk(s0, 0);
      mask_chunk(s1, 1);
      mask_chunk(s2, 2);
      mask_chunk(s3, 3);
#pragma unroll
      for (int e = 0; e < 32; ++e)
        m4[e & 3] = fmaxf(m4[e & 3], fmaxf(fmaxf(__uint_as_float(s0[e]), __uint_as_float(s1[e])),
                                           fmaxf(__uint_as_float(s2[e]), __uint_as_float(s3[e]))));
      // max of the raw scores (scale > 0 commutes with max)
      const float mraw = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
      const float mx = mraw * args.sl2;
      const float m_new = (mx > m_used + 8.f) ? mx : m_used;
      const float alpha = (m_new != m_used) ? fast_exp2(m_used - m_new) : 1.f;
      const float mb = (m_new == -INFINITY) ? 0.f : m_new;
      // pass 2: P as bf16 pairs, 32 keys -> 16 TMEM columns at a time, written
      // over the first 64 columns of S (every score is already in registers);
      // four independent partial sums
      float r4[4] = {0.f, 0.f, 0.f, 0.f};
      // EMU of every 16 exponentials go to the FMA pipe on unmasked tiles (masked
      // -inf scores need the exact 0 of ex2)
      const bool emu = EMU > 0 && !need_mask;
      if (SEP && jj > 0) {
        // P(jj-1) in the P columns must have been read by its PV MMA
        w_ok = bounded_wait(o_done + 8 * t, (jj - 1) & 1, args.status, LK_ERR_TIMEOUT_ACCUM, abort_flag);
        if (!__all_sync(0xffffffffu, w_ok)) {
          ok = false;
          break;
        }
        tc_fence_after();
      }
      auto emit = [&](const uint32_t (&x)[32], int c) {
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          const float a0 = fmaf(__uint_as_float(x[e]), args.sl2, -mb);
          const float a1 = fmaf(__uint_as_float(x[e + 1]), args.sl2, -mb);
          const float p0 = fast_exp2(a0);
          float p1;
          if (((e >> 1) & 7) < EMU) {
            p1 = emu ? exp2_fma(a1) : fast_exp2(a1);
          } else {
            p1 = fast_exp2(a1);
          }
          r4[(e >> 1) & 3] += p0 + p1;
          pk[e >> 1] = pack_bf16x2(p0, p1);
        }
        tmem_st16(tP + c * 16, pk);
      };
      emit(s0, 0);
      emit(s1, 1);
      emit(s2, 2);
      emit(s3, 3);
      const float rowsum = (r4[0] + r4[1]) + (r4[2] + r4[3]);
      // rescale O (rare): PV(jj-1) must have finished accumulating
      if (jj > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
        w_ok = bounded_wait(o_done + 8 * t, (jj - 1) & 1, args.status, LK_ERR_TIMEOUT_ACCUM, abort_flag);
        if (!__all_sync(0xffffffffu, w_ok)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < DH / 32; ++c) {
          uint32_t ov[32];
          tmem_ld32(tO + c * 32, ov);
          tc_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) ov[e] = __float_as_uint(__uint_as_float(ov[e]) * alpha);
          tmem_st32(tO + c * 32, ov);
        }
      }
      tc_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full + 8 * t);
      l_run = l_run * alpha + rowsum;
      m_used = m_new;
    }
    if (ok && n_t > 0) {
      bool w_ok = bounded_wait(o_done + 8 * t, (n_t - 1) & 1, args.status, LK_ERR_TIMEOUT_ACCUM, abort_flag);
      if (__all_sync(0xffffffffu, w_ok)) {
        tc_fence_after();
        const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
        __nv_bfloat16* orow = args.o + (int64_t)(row0 + ql) * args.ldo + h * DH;
#pragma unroll 1
        for (int c = 0; c < DH / 32; ++c) {
          uint32_t v[32];
          tmem_ld32(tO + c * 32, v);
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
  a.n_qtiles = cdiv(d.S, 256);  // pairs of 128-query tiles, one per CTA
  static const int emu = [] {
    const char* e = getenv("LK_ATTN_EXP_EMU");
    return e ? atoi(e) : 0;
  }();
  // LK_ATTN_SPLIT=1: two threads per query row (16 softmax warps)
  static const int split = [] {
    const char* e = getenv("LK_ATTN_SPLIT");
    return (e && atoi(e) == 1) ? 2 : 1;
  }();
  a.emu = emu;
  auto k = split == 2 ? attn_fwd_kernel<DH, 0, 2>
                      : (a.emu >= 4 ? attn_fwd_kernel<DH, 4, 1>
                                    : a.emu >= 2 ? attn_fwd_kernel<DH, 2, 1> : attn_fwd_kernel<DH, 0, 1>);
  cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  k<<<a.n_qtiles * d.Hq * d.B, C::threads(split), C::SMEM, s>>>(tm, tkv, a);
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
