// Plain C ABI of the lora_kernel_b200 CUDA library.
//
// Every launcher takes raw device pointers, sizes and strides plus the CUDA
// stream, enqueues its kernel(s) and returns 0 on success or -1 with a message
// retrievable through lk_last_error().  The torch bindings (bindings.cpp)
// validate tensors and call these; C/C++ callers can use them directly.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

const char* lk_last_error(void);
// Kernels enqueued by this library so far (for launch accounting).
unsigned long long lk_launch_count(void);

// ------------------------------------------------------------------ K1 GEMM
// D[M,N] = alpha * A[M,K] . B[N,K]^T with a fused epilogue.  Operands are
// described by their physical row-major storage: a K-major operand X[rows,K]
// is stored [rows, K] (x_mn = 0); an MN-major one is stored [K, rows] (x_mn = 1).
enum LkGemmEpi {
  LK_EPI_BF16 = 0,
  LK_EPI_F32 = 1,
  LK_EPI_F32_ACC = 2,
  LK_EPI_BF16_RESID = 3,
  LK_EPI_SWIGLU = 4,
  LK_EPI_REMOTE = 5,
  // SwiGLU backward fused into the GEMM that produces dh = dL/d(silu(g) u):
  // d is the bf16 gate|up gradient [M, 2N] (128-column blocks, pitch ldd) and r
  // the forward gate|up activation in the same layout (pitch ldr); dh itself is
  // not stored
  LK_EPI_SWIGLU_BWD = 6,
  // bf16 output whose first rope_cols columns are rotary-embedded on the way
  // out: heads of width rope_dh, interleaved pairs (2i, 2i+1), row m at position
  // m % rope_seq + rope_off, (cos, sin) from rope_table float2 [max_pos, rope_dh/2]
  LK_EPI_BF16_ROPE = 7,
};

typedef struct LkGemmDesc {
  const void* a;
  int64_t a_rows, a_cols, a_ld;
  int a_mn;
  const void* b;
  int64_t b_rows, b_cols, b_ld;
  int b_mn;
  int M, N, K;
  void* d;
  int64_t ldd;
  const void* r;  // residual (LK_EPI_BF16_RESID)
  int64_t ldr;
  void* h;  // silu(gate)*up output (LK_EPI_SWIGLU)
  int64_t ldh;
  float alpha;
  int epi;
  int bn;  // 0 = choose, 128 or 256
  int* status;
  // Optional second contraction segment accumulated into the same output:
  // D = alpha * (A.B^T + A2.B2^T); A2 [M, K2] and B2 [N, K2] share the majorness
  // of A and B (used by the fused LoRA update: A2 = s*x*A_lora^T, B2 = B_lora).
  const void* a2;
  int64_t a2_rows, a2_cols, a2_ld;
  const void* b2;
  int64_t b2_rows, b2_cols, b2_ld;
  int K2;
  // Fused collectives (comm_mode): 0 none; 1 = K18 GEMM -> reduce-scatter: the
  // bf16 output row m goes to rank m / rs_rows at row (rs_rank * rs_rows + m %
  // rs_rows) of its receive buffer rptrs[owner] (pitch ldd; rptrs is a DEVICE
  // array of peer pointers); 2 = K16 all-gather -> GEMM: A (K-major, [M, K],
  // any local buffer) is filled on first use from ag_src[p] (DEVICE array of
  // pointers to each rank's ag_rows x K staging rows in symmetric memory,
  // pitch ag_ld_src bytes, this rank's own entry included); ag_count is int
  // scratch [M/128] zeroed by the launcher.  m_rot rotates the M-tile order.
  int comm_mode;
  int m_rot;
  void* const* rptrs;
  const void* rmaps;  // optional K18 TMA stores: DEVICE array of per-owner tensor maps (lk_make_remote_maps)
  int rs_rows, rs_rank;
  const void* const* ag_src;
  int64_t ag_ld_src;
  int ag_rows, ag_rank, ag_world;
  int* ag_count;
  // 3 = K17 ZeRO-3 group gather -> GEMM: the flat parameter group (gb_len
  // elements, bf16) is assembled at gb_dst from the owners' chunks gb_src[p]
  // (DEVICE array of `ag_world` pointers, gb_chunk elements each) by the GEMM's
  // copy warps; B must be the [N, K] view at element gb_boff of gb_dst.
  // gb_count: int scratch [ceil(N / 128)] zeroed by the launcher.  ag_rank
  // rotates the copy order.
  const void* const* gb_src;
  int64_t gb_chunk, gb_len, gb_boff;
  void* gb_dst;
  int* gb_count;
  // LK_EPI_BF16_ROPE
  const void* rope_table;
  int rope_cols, rope_dh, rope_seq, rope_off;
} LkGemmDesc;

int lk_gemm(const LkGemmDesc* desc, cudaStream_t stream);
// CTA-pair tiles (tcgen05.mma.cta_group::2, 256 x 256) for plain GEMMs: 0 off, 1 on
// (the default; LK_GEMM_PAIR in the environment at the first GEMM overrides it)
void lk_gemm_set_pair(int mode);
unsigned long long lk_gemm_pair_count(void);  // GEMMs that took the CTA-pair path so far
// Encode the K18 store tensor maps of `world` receive buffers (bf16 [rows, cols],
// pitch ld elements; 32 x 64 boxes, 128-byte swizzle) into host memory out
// (world * 128 bytes, to be copied to the device by the caller).
int lk_make_remote_maps(void* const* host_ptrs, int world, int64_t rows, int64_t cols, int64_t ld, void* out);

// --------------------------------------------------------------- K5 RMSNorm
typedef struct LkNormFwdDesc {
  const void* x;    // [M, D] bf16
  const void* res;  // optional residual [M, D] bf16 (h = x + res)
  const void* gamma;
  void* y;          // [M, D] bf16
  void* h_out;      // [M, D] bf16 when res != NULL (may alias x)
  float* rstd;      // [M] fp32 (may be NULL)
  int M, D;
  float eps;
} LkNormFwdDesc;

typedef struct LkNormBwdDesc {
  const void* dy;     // [M, D] bf16
  const void* x;      // normalised input h [M, D] bf16
  const void* gamma;  // [D] bf16
  const float* rstd;  // [M]
  const void* dres;   // optional gradient to add (may alias dx)
  void* dx;           // [M, D] bf16
  float* dgamma;      // [D] fp32
  float* partial;     // scratch [partial_rows, D] fp32
  int partial_rows;
  int M, D;
  int accumulate;     // dgamma += (1) or = (0)
  int dgamma_bf16;    // 1: dgamma points to bf16 [D] and is stored (accumulate must be 0)
} LkNormBwdDesc;

int lk_rmsnorm_fwd(const LkNormFwdDesc* d, cudaStream_t s);
int lk_rmsnorm_bwd(const LkNormBwdDesc* d, cudaStream_t s);
int lk_rmsnorm_bwd_partial_rows(int M);

// ------------------------------------------------------------------ K6 RoPE
typedef struct LkRopeDesc {
  void* x;            // bf16 [T, ...] row pitch ld
  int64_t ld;
  int T, col0, nheads, Dh;
  const void* table;  // float2 [max_pos, Dh/2] (cos, sin)
  const int* pos;     // optional per-token positions
  int seq_len, pos_offset;
  int inverse;
} LkRopeDesc;
int lk_rope(const LkRopeDesc* d, cudaStream_t s);

// ------------------------------------------------------ K7 SwiGLU, K8 embedding
int lk_swiglu_fwd(const void* gu, void* h, int M, int F, cudaStream_t s);
int lk_swiglu_bwd(const void* gu, const void* dh, void* dgu, int M, int F, cudaStream_t s);
int lk_cast_f32_bf16(const float* x, void* y, int64_t n, cudaStream_t s);
int lk_embedding_fwd(const int64_t* ids, const void* W, void* out, int T, int D, int V,
                     int* status, cudaStream_t s);
int lk_embedding_bwd(const int64_t* ids, const void* dy, float* dW, int T, int D, int V,
                     cudaStream_t s);

// ------------------------------------------------- K2 block-scaled fp8 GEMM
// D[M, N] (bf16) = (A8 . B8^T with per-block scales) [+ R].  A8 [M, K] fp8
// (a_fmt 0 = e4m3, 1 = e5m2), scale sa[K/128][M] (one per row and 128-wide K
// block); B8 [N, K] e4m3, scale sb[ceil(N/128)][K/128] (one per 128 x 128
// block).  K % 128 == 0; pitches in elements (= bytes) multiples of 16.
typedef struct LkGemmFp8Desc {
  const void* a;
  int64_t a_ld;
  const void* b;
  int64_t b_ld;
  int M, N, K, a_fmt;
  const float* sa;
  const float* sb;
  void* d;
  int64_t ldd;
  const void* r;  // optional residual (bf16, pitch ldr)
  int64_t ldr;
  int* status;
  // Fused collectives (at most one): all-gather of A on first use - every
  // rank's ag_rows_per_rank fp8 rows (ag_rows[p], pitch K) and scales
  // (ag_scales[p], [K/128][ag_rows_per_rank]) are copied into a / sa (DEVICE
  // pointer arrays of `world` entries; ag_count int scratch [M/128]); or
  // reduce-scatter epilogue - bf16 row m goes to rptrs[m / rs_rows] at row
  // rank * rs_rows + m % rs_rows (pitch ldd).
  const void* const* ag_rows;
  const float* const* ag_scales;
  int ag_rows_per_rank;
  int* ag_count;
  void* const* rptrs;
  int rs_rows;
  int rank, world;
} LkGemmFp8Desc;
int lk_gemm_fp8(const LkGemmFp8Desc* desc, cudaStream_t stream);
// x bf16 [M, K] -> q fp8 [M, K] (fmt 0 e4m3 / 1 e5m2) + scale [K/128][M]
int lk_quant_1x128(const void* x, int64_t ldx, int M, int K, int fmt, void* q, int64_t ldq, float* scale,
                   cudaStream_t s);
// q fp8 [M, K] with scale [K/128][M] -> x bf16 [M, ldx]
int lk_dequant_1x128(const void* q, int M, int K, int fmt, const float* scale, void* x, int64_t ldx, cudaStream_t s);
// w bf16 [N, K] -> q e4m3 [N, K], optional qt = q^T [K, N], scale [ceil(N/128)][K/128]
int lk_quant_128x128(const void* w, int64_t ldw, int N, int K, void* q, void* qt, float* scale, cudaStream_t s);

// ----------------------------------- K2, MX form: hardware block-scaled fp8 GEMM
// D[M, N] (bf16) = sum_k 2^ea[m, k/32] 2^eb[n, k/32] A8[m, k] B8[n, k] [+ R].
// A8 [M, K], B8 [N, K] fp8 bits (fmt 0 e4m3, 1 e5m2), K % 128 == 0.  Scales are
// UE8M0 bytes in "SF tiles": an operand of R rows has ceil(R/128) x K/128 tiles
// of 512 bytes, tile (rt, kb) at (rt K/128 + kb) 512, row r / 32-wide block j at
// (r % 32) 16 + ((r % 128) / 32) 4 + j inside it.  sfa covers ceil(M/128) row
// tiles, sfb 2 ceil(N/256) (rows past N: any finite exponent).
typedef struct LkGemmMxf8Desc {
  const void* a;
  int64_t a_ld;
  const void* b;
  int64_t b_ld;
  int M, N, K, a_fmt, b_fmt;
  const void* sfa;
  const void* sfb;
  void* d;
  int64_t ldd;
  const void* r;  // optional residual (bf16, pitch ldr)
  int64_t ldr;
  int* status;
  // Fused collectives (at most one, e4m3 operands): all-gather of A - every
  // rank's ag_rows_per_rank rows (ag_rows[p], pitch K) and SF tiles (ag_sf[p])
  // are copied into a / sfa (DEVICE pointer arrays of `world` entries; ag_count
  // int scratch [M/128]); or reduce-scatter epilogue - bf16 row m goes to
  // rptrs[m / rs_rows] at row rank * rs_rows + m % rs_rows (pitch ldd).
  const void* const* ag_rows;
  const void* const* ag_sf;
  int ag_rows_per_rank;
  int* ag_count;
  void* const* rptrs;
  int rs_rows;
  int rank, world;
} LkGemmMxf8Desc;
int lk_gemm_mxf8(const LkGemmMxf8Desc* desc, cudaStream_t stream);
// x bf16 [M, K] -> q fp8 [M, K] with one power-of-two scale per row and 128-wide
// K block (UE8M0 SF tiles over rows_pad rows; rows >= M get exponent 0)
int lk_quant_mx_rows(const void* x, int64_t ldx, int M, int rows_pad, int K, int fmt, void* q, int64_t ldq,
                     void* sf, cudaStream_t s);
// w bf16 [N, K] -> q e4m3 [N, K] with one power-of-two scale per 128 x 128 block:
// SF tiles sf (ceil(N/128) row tiles), fp32 scales [ceil(N/128)][K/128], and
// optionally qt = q^T [K, N] with its SF tiles sft (K/128 row tiles x N/128)
int lk_quant_mx_128x128(const void* w, int64_t ldw, int N, int K, void* q, void* sf, float* scale, void* qt,
                        void* sft, cudaStream_t s);
// q fp8 [M, K] with SF tiles -> x bf16 [M, ldx]
int lk_dequant_mx_rows(const void* q, int M, int K, int fmt, const void* sf, void* x, int64_t ldx, cudaStream_t s);

// --------------------------------------------- K18 owner-side slot reduction
typedef struct LkRsSumDesc {
  const void* recv;   // [world * rows, ld_recv] bf16: slot s = rank s's partial
  int64_t ld_recv;
  int world, rows, cols;
  const void* resid;  // optional [rows, ld_resid] bf16 added to the sum
  int64_t ld_resid;
  void* out;          // [rows, ld_out] bf16 sum (may alias resid)
  int64_t ld_out;
  const void* gamma;  // optional: RMSNorm of the sum -> y, rstd
  void* y;
  int64_t ld_y;
  float* rstd;
  float eps;
  // Source of the partial sums (the RMSNorm form only): 0 = `world` slots of
  // recv (K18 owner side); 1 = all-reduce: row r of every rank's own partial
  // buffer peers[s] (DEVICE array of `world` pointers, pitch ld_recv); 2 =
  // all-reduce through the buffer's NVLS multicast address `mc`.
  int src_mode;
  const void* const* peers;
  const void* mc;
} LkRsSumDesc;
int lk_rs_sum(const LkRsSumDesc* d, cudaStream_t s);

// ------------------------------------------- GELU (tanh form) and LayerNorm
int lk_gelu_fwd(const void* x, void* y, int64_t n, cudaStream_t s);
int lk_gelu_bwd(const void* x, const void* dy, void* dx, int64_t n, cudaStream_t s);
int lk_dropout(const void* x, void* y, int64_t n, float p, uint64_t seed, cudaStream_t s);
// y = (x - mean) * rstd * gamma + beta (bf16 [M, D], D = 256 x {1,2,4,8,16}); mean / rstd fp32 [M]
int lk_layernorm_fwd(const void* x, const void* gamma, const void* beta, void* y, float* mean, float* rstd,
                     int M, int D, float eps, cudaStream_t s);
// dx (bf16); dgamma / dbeta (fp32 [D]) are ADDED to
int lk_layernorm_bwd(const void* dy, const void* x, const void* gamma, const float* mean, const float* rstd,
                     void* dx, float* dgamma, float* dbeta, int M, int D, cudaStream_t s);

// ------------------------------------------------------------ K9 cross-entropy
typedef struct LkCeDesc {
  void* logits;  // [T, V] bf16, overwritten with the gradient when write_grad
  int64_t ld;
  const int64_t* targets;
  int T, V;
  float* loss_acc;        // [2]: += sum of losses, += number of counted rows
  float* row_loss;        // optional [T]
  const float* scale_ptr; // optional device scalar (loss scale)
  float scale_mul;
  float smoothing, zloss;
  int64_t ignore_index;
  int write_grad;
} LkCeDesc;
int lk_cross_entropy(const LkCeDesc* d, cudaStream_t s);

// Vocabulary-parallel cross-entropy: each rank holds logits [T, V_local] for
// vocabulary columns [v0, v0 + V_local).  Phase 1 writes per-row partial
// statistics {max, sum exp, sum z, z[target] if owned} to stats (float4 [T],
// symmetric memory); after a device barrier phase 2 combines every rank's
// statistics (peer pointers `peer_stats`, a DEVICE array of `world` float4*)
// into the loss (identical on every rank) and writes the local dlogits slice.
typedef struct LkCeVpDesc {
  LkCeDesc ce;         // logits / ld / targets / T / V (= V_local) / loss / scale fields
  int64_t v0, V_total;
  float* stats;        // this rank's float4 [T]
  const float* const* peer_stats;
  int world, phase;
} LkCeVpDesc;
int lk_cross_entropy_vp(const LkCeVpDesc* d, cudaStream_t s);

// ------------------------------------------------------- K11 AdamW + K12 (1 GPU)
// Device-resident optimizer state vector (fp32) indices.
enum LkOptState {
  LK_ST_LOSS_SCALE = 0,
  LK_ST_GROWTH_TRACKER = 1,
  LK_ST_STEP = 2,
  LK_ST_GRAD_MULT = 3,
  LK_ST_SKIP = 4,
  LK_ST_LR = 5,
  LK_ST_GRAD_NORM = 6,
  LK_ST_NUM_SKIPPED = 7,
  LK_ST_CONSEC_SKIPS = 8,
  LK_ST_CLIP_COEF = 9,
  LK_ST_SIZE = 16,
};

typedef struct LkAdamWDesc {
  float *p32, *g, *m, *v;
  void* p16;        // optional bf16 copy of the params
  float* ema;       // optional EMA of the params
  const int* chunks;  // int4 [nchunks]: start, length, wd on/off, 0
  int nchunks;
  const float* state;
  float beta1, beta2, eps, wd, ema_decay;
  int zero_grad;
  // Optional fused parameter all-gather (ZeRO-1/2): the new bf16 value of
  // master element o is also stored into every rank's full parameter buffer
  // (p16_peers, a DEVICE array of `world` bf16 pointers) at element
  // o + 64 * chunks[c].w, the chunk's shard-to-flat offset in 64-element units.
  void* const* p16_peers;
  int world;
} LkAdamWDesc;
int lk_adamw(const LkAdamWDesc* d, cudaStream_t s);
int lk_grad_norm_partials(const float* g, int64_t n, float* partial, int nparts, cudaStream_t s);
int lk_optimizer_finalize(const float* partial, int nparts, float* state, float max_norm,
                          int dynamic, float growth, float backoff, int growth_interval,
                          float min_scale, cudaStream_t s);

// ------------------------------------------------------- K3/K4 flash attention
typedef struct LkAttnDesc {
  const void* qkv;  // [B*S, (Hq+2Hkv)*Dh] bf16, row pitch ld_qkv
  int64_t ld_qkv;
  void* o;          // [B*S, Hq*Dh] bf16, row pitch ld_o
  int64_t ld_o;
  float* lse;       // [B, Hq, S] natural-log LSE
  int B, S, Hq, Hkv, Dh;
  int causal, window;
  float scale;
  int* status;
  // Optional separate key/value source (serving prefill over a cached prefix):
  // when kv != NULL, qkv holds only the queries [B*S, Hq*Dh] and kv holds
  // [B*Skv, 2*Hkv*Dh] (keys then values); query i sits at position q_off + i.
  const void* kv;
  int64_t ld_kv;
  int Skv, q_off;
} LkAttnDesc;
int lk_attention_fwd(const LkAttnDesc* d, cudaStream_t s);

typedef struct LkAttnBwdDesc {
  const void* qkv;
  int64_t ld_qkv;
  const void* o;
  int64_t ld_o;
  const void* dout;  // [B*S, Hq*Dh]
  int64_t ld_do;
  const float* lse;
  void* dqkv;        // [B*S, (Hq+2Hkv)*Dh] bf16 output
  int64_t ld_dqkv;
  float* dq_acc;     // scratch [B*S, Hq*Dh] fp32
  float* dvec;       // scratch fp32: 2 x round_up(B*Hq*S, 64) (scaled D, LSE * log2(e))
  int B, S, Hq, Hkv, Dh;
  int causal, window;
  float scale;
  int* status;
} LkAttnBwdDesc;
int lk_attention_bwd(const LkAttnBwdDesc* d, cudaStream_t s);

// ------------------------------------------- K15 KV append / K13 decode / K19
typedef struct LkKvAppendDesc {
  const void* qkv;  // [T, (Hq+2Hkv)*Dh] bf16 (post-RoPE), row pitch ld
  int64_t ld;
  int T, Hq, Hkv, Dh;
  const int* slots;  // [T] block_id * block_size + offset, < 0 = skip
  void* k_cache;     // [num_slots, Hkv, Dh]
  void* v_cache;
  float* k_scale;    // [num_slots, Hkv] (quantized caches)
  float* v_scale;
  int num_slots;
  int kv_dtype;      // 0 bf16, 1 fp8 e4m3, 2 int8
  int* status;
} LkKvAppendDesc;
int lk_kv_append(const LkKvAppendDesc* d, cudaStream_t s);

typedef struct LkDecodeDesc {
  const void* q;  // [num_seqs, Hq*Dh] bf16, row pitch ldq
  int64_t ldq;
  const void* k_cache;
  const void* v_cache;
  const float* k_scale;
  const float* v_scale;
  const int* block_tables;  // [num_seqs, max_blocks]
  int max_blocks;
  const int* ctx_lens;      // [num_seqs]
  int block_size, num_seqs, Hq, Hkv, Dh;
  float scale;
  int split_len, num_splits;
  float* part_o;   // [num_seqs, Hq, num_splits, Dh] when num_splits > 1
  float* part_ml;  // [num_seqs, Hq, num_splits, 2]
  void* out;       // [num_seqs, Hq*Dh] bf16
  int64_t ldo;
  int kv_dtype;
  int num_blocks;  // physical KV blocks (bounds-checked builds verify block-table entries)
  int* status;     // optional device status word
} LkDecodeDesc;
int lk_decode_attention(const LkDecodeDesc* d, cudaStream_t s);
int lk_kv_gather(const void* k_cache, const void* v_cache, const float* k_scale, const float* v_scale,
                 const int* slots, int n, int Hkv, int Dh, void* out, int64_t ldo, int kv_dtype,
                 cudaStream_t s);
// Same, with the cache's slot count and a status word: bounds-checked builds
// verify every slot and record an out-of-range one there (its row is zeroed).
int lk_kv_gather_checked(const void* k_cache, const void* v_cache, const float* k_scale, const float* v_scale,
                         const int* slots, int n, int Hkv, int Dh, void* out, int64_t ldo, int kv_dtype,
                         int num_slots, int* status, cudaStream_t s);
int lk_sample(const void* logits, int64_t ld, int rows, int V, const float* temperature,
              uint64_t seed, int64_t* out_tok, float* out_val, cudaStream_t s);
int lk_sample_vp(const void* logits, int64_t ld, int rows, int V, int64_t v0, const float* temperature,
                 uint64_t seed, int64_t* out_tok, float* out_val, cudaStream_t s);
// Nucleus sampling (one GPU): per-row temperature and top_p (rows with top_p >= 1
// or temperature <= 0 behave as lk_sample); optional per-row seeds (nullptr:
// the noise of lk_sample for `seed`).
int lk_sample_topp(const void* logits, int64_t ld, int rows, int V, const float* temperature,
                   const float* top_p, uint64_t seed, const uint64_t* row_seeds, int64_t* out_tok,
                   cudaStream_t s);

// ------------------------------------------------------ K14 quantised weights
enum LkQuantFmt { LK_Q_INT8 = 0, LK_Q_FP8 = 1, LK_Q_INT4 = 2 };
int lk_quantize(int fmt, const void* w, int N, int K, int group, void* q, float* scale, float* zero,
                cudaStream_t s);
int lk_dequant_gemv(int fmt, const void* x, int64_t ldx, int M, const void* q, const float* scale,
                    const float* zero, int N, int K, int group, void* y, int64_t ldy, cudaStream_t s);
int lk_dequantize(int fmt, const void* q, const float* scale, const float* zero, int N, int K,
                  int group, void* w, cudaStream_t s);
// Weight-streaming dequant GEMM for decode batches (tcgen05, 1 <= M <= 256):
// y[M, N] (bf16) = x[M, K] (bf16, pitch ldx) . dequant(q)^T (+ r).  q / scale /
// zero in the lk_quantize layouts (int4: K % 64 == 0, group % 64 == 0).  With
// splits > 1 (0 = lk_dq_gemm_splits) each split writes an fp32 partial to
// partial [splits, M, N], summed in split order into y.
typedef struct LkDqGemmDesc {
  int fmt;
  const void* x;
  int64_t ldx;
  int M;
  const void* q;
  const float* scale;
  const float* zero;
  int N, K, group;
  void* y;
  int64_t ldy;
  const void* r;
  int64_t ldr;
  float* partial;
  int splits;
  int* status;
  // optional: LK_DQ_COUNTERS int32 zeros, one per 128-row weight tile; with it the
  // last split of each tile sums the partials in the same launch (else a second
  // kernel does); the kernel leaves them zero again
  int* counters;
} LkDqGemmDesc;
#define LK_DQ_COUNTERS 16384
int lk_dq_gemm(const LkDqGemmDesc* d, cudaStream_t s);
int lk_dq_gemm_splits(int M, int N, int K);

// ---------------------------------------------- peer-memory collectives (comm.cu)
// Pointer arguments named *_ptrs are DEVICE arrays of `world` peer pointers
// (rank order) into symmetric (peer-mapped) buffers.  Flag arrays hold
// LK_SIG_SLOTS * world int32 per rank, zero-initialised; epochs increase.
#define LK_SIG_SLOTS 16
// Device-epoch form (graph-replayable): *epoch_ctr (device int) is advanced by the kernel.
int lk_signal_barrier_dev(int* const* sig_ptrs, int rank, int world, int slot, int* epoch_ctr, int* status,
                          cudaStream_t s);
int lk_signal_barrier(int* const* sig_ptrs, int rank, int world, int slot, int epoch, int* status,
                      cudaStream_t s);
int lk_allgather_copy(const void* const* src_ptrs, int64_t src_off_bytes, int64_t chunk_bytes,
                      void* dst, int world, cudaStream_t s);
int lk_reduce_scatter_sum(const float* const* src_ptrs, int64_t src_off, int64_t n, float* dst,
                          int world, int accumulate, float* partial, int nparts, cudaStream_t s);
// NVLS variants: `mc` is the multicast address of the symmetric buffer (+ the
// element offset); reductions happen inside the NVSwitch (multimem.*).
int lk_allreduce_sum_nvls(float* mc, int64_t n, int rank, int world, float* partial, int nparts,
                          cudaStream_t s);
int lk_reduce_scatter_sum_nvls(const float* mc, int64_t n, float* dst, int accumulate, float* partial,
                               int nparts, cudaStream_t s);
// bf16 gradients in, fp32 shard out (+= when accumulate), Σg² partials of the shard
int lk_reduce_scatter_bf16(const void* const* src_ptrs, int64_t src_off, int64_t n, float* dst, int world,
                           int accumulate, float* partial, int nparts, cudaStream_t s);
int lk_reduce_scatter_bf16_nvls(const void* mc, int64_t n, float* dst, int accumulate, float* partial,
                                int nparts, cudaStream_t s);
int lk_allreduce_sum(float* const* buf_ptrs, int64_t n, int rank, int world, float* partial,
                     int nparts, cudaStream_t s);
int lk_norm_exchange(const float* partial, int nparts, double* const* nbuf_ptrs, int* const* sig_ptrs,
                     int rank, int world, int slot, int epoch, float* state, float max_norm,
                     int dynamic, float growth, float backoff, int growth_interval, float min_scale,
                     int* status, cudaStream_t s);

#ifdef __cplusplus
}
#endif
