// Torch bindings of the lora_kernel_b200 CUDA library (module lora_kernel_b200._C).
// Each binding checks devices/dtypes/shapes, fills the C descriptor and calls
// the launcher on the current CUDA stream; launcher errors become Python
// RuntimeErrors.  No binding falls back to another implementation.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "lk_api.h"

namespace {

cudaStream_t stream() { return at::cuda::getCurrentCUDAStream().stream(); }

void check(int rc) { TORCH_CHECK(rc == 0, "lora_kernel_b200: ", lk_last_error()); }

void need(const torch::Tensor& t, const char* name, c10::ScalarType dt) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.scalar_type() == dt, name, " has dtype ", t.scalar_type(), ", expected ", dt);
}

void need_contig(const torch::Tensor& t, const char* name, c10::ScalarType dt) {
  need(t, name, dt);
  TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
}

template <typename T = void>
T* optp(const c10::optional<torch::Tensor>& t) {
  return t.has_value() && t->defined() ? reinterpret_cast<T*>(t->data_ptr()) : nullptr;
}

// ----------------------------------------------------------------- GEMM
struct Operand {
  const void* base;
  int64_t rows, cols, ld;
  int mn;
};

Operand classify(const torch::Tensor& x, const char* name) {
  need(x, name, torch::kBFloat16);
  TORCH_CHECK(x.dim() == 2, name, " must be 2-D");
  Operand o;
  o.base = x.data_ptr();
  const int64_t r = x.size(0), k = x.size(1);
  if (x.stride(1) == 1 && (r == 1 || x.stride(0) >= k)) {
    o.mn = 0;
    o.rows = r;
    o.cols = k;
    o.ld = r == 1 ? ((k + 7) / 8) * 8 : x.stride(0);
  } else if (x.stride(0) == 1 && (k == 1 || x.stride(1) >= r)) {
    o.mn = 1;
    o.rows = k;
    o.cols = r;
    o.ld = k == 1 ? ((r + 7) / 8) * 8 : x.stride(1);
  } else {
    TORCH_CHECK(false, name, " needs a unit stride in one dimension");
  }
  return o;
}

void gemm(torch::Tensor a, torch::Tensor b, torch::Tensor out, int64_t epi,
          c10::optional<torch::Tensor> resid, c10::optional<torch::Tensor> h, double alpha,
          torch::Tensor status, int64_t bn, c10::optional<torch::Tensor> a2,
          c10::optional<torch::Tensor> b2, c10::optional<torch::Tensor> rope_table, int64_t rope_cols,
          int64_t rope_dh, int64_t rope_seq, int64_t rope_off) {
  const c10::cuda::CUDAGuard g(a.device());
  TORCH_CHECK(a.size(1) == b.size(1), "gemm: K mismatch ", a.sizes(), " vs ", b.sizes());
  Operand A = classify(a, "a"), B = classify(b, "b");
  LkGemmDesc d{};
  d.a = A.base; d.a_rows = A.rows; d.a_cols = A.cols; d.a_ld = A.ld; d.a_mn = A.mn;
  d.b = B.base; d.b_rows = B.rows; d.b_cols = B.cols; d.b_ld = B.ld; d.b_mn = B.mn;
  d.M = (int)a.size(0);
  d.N = (int)b.size(0);
  d.K = (int)a.size(1);
  // the SwiGLU-backward epilogue writes gate|up gradients: [M, 2N]
  const int64_t out_cols = epi == LK_EPI_SWIGLU_BWD ? 2 * (int64_t)d.N : d.N;
  TORCH_CHECK(out.is_cuda() && out.dim() == 2 && out.size(0) == d.M && out.size(1) == out_cols &&
                  out.stride(1) == 1,
              "gemm: out must be row-major [M, N] ([M, 2N] for swiglu_bwd)");
  const bool f32 = epi == LK_EPI_F32 || epi == LK_EPI_F32_ACC;
  TORCH_CHECK(out.scalar_type() == (f32 ? torch::kFloat32 : torch::kBFloat16), "gemm: out dtype");
  d.d = out.data_ptr();
  d.ldd = out.stride(0);
  if (resid.has_value()) {
    need(*resid, "resid", torch::kBFloat16);
    TORCH_CHECK(resid->size(0) == d.M && resid->size(1) == out_cols && resid->stride(1) == 1, "gemm: resid shape");
    d.r = resid->data_ptr();
    d.ldr = resid->stride(0);
  }
  if (h.has_value()) {
    need(*h, "h", torch::kBFloat16);
    TORCH_CHECK(h->size(0) == d.M && h->size(1) == d.N / 2 && h->stride(1) == 1, "gemm: h shape");
    d.h = h->data_ptr();
    d.ldh = h->stride(0);
  }
  d.alpha = (float)alpha;
  d.epi = (int)epi;
  d.bn = (int)bn;
  if (rope_table.has_value()) {
    need_contig(*rope_table, "rope_table", torch::kFloat32);
    TORCH_CHECK(epi == LK_EPI_BF16_ROPE && rope_table->dim() == 3 && rope_table->size(1) * 2 == rope_dh,
                "gemm: rope table [max_pos, Dh/2, 2] with the rope epilogue");
    TORCH_CHECK(rope_seq + rope_off <= rope_table->size(0), "gemm: rope positions beyond the table");
    d.rope_table = rope_table->data_ptr();
    d.rope_cols = (int)rope_cols;
    d.rope_dh = (int)rope_dh;
    d.rope_seq = (int)rope_seq;
    d.rope_off = (int)rope_off;
  } else {
    TORCH_CHECK(epi != LK_EPI_BF16_ROPE, "gemm: the rope epilogue needs its table");
  }
  need(status, "status", torch::kInt32);
  d.status = status.data_ptr<int>();
  if (a2.has_value() && b2.has_value()) {
    TORCH_CHECK(a2->size(0) == d.M && b2->size(0) == d.N && a2->size(1) == b2->size(1),
                "gemm: second segment shapes");
    Operand A2 = classify(*a2, "a2"), B2 = classify(*b2, "b2");
    TORCH_CHECK(A2.mn == A.mn && B2.mn == B.mn, "gemm: segment operands must share majorness");
    d.a2 = A2.base; d.a2_rows = A2.rows; d.a2_cols = A2.cols; d.a2_ld = A2.ld;
    d.b2 = B2.base; d.b2_rows = B2.rows; d.b2_cols = B2.cols; d.b2_ld = B2.ld;
    d.K2 = (int)a2->size(1);
  }
  check(lk_gemm(&d, stream()));
}

// K18: GEMM whose bf16 output rows are stored into their owner rank's receive
// buffer (peer pointers `rptrs`, int64 device tensor) at slot rs_rank.
// Device copy of the K18 store tensor maps of every rank's receive buffer.
torch::Tensor make_remote_maps(std::vector<int64_t> ptrs, int64_t rows, int64_t cols, int64_t ld,
                               torch::Device device) {
  std::vector<void*> p(ptrs.size());
  for (size_t i = 0; i < ptrs.size(); ++i) p[i] = reinterpret_cast<void*>(ptrs[i]);
  auto host = torch::empty({(int64_t)ptrs.size() * 128}, torch::dtype(torch::kUInt8));
  check(lk_make_remote_maps(p.data(), (int)p.size(), rows, cols, ld, host.data_ptr()));
  return host.to(device);
}

void gemm_rs(torch::Tensor a, torch::Tensor b, torch::Tensor rptrs, int64_t rs_rows, int64_t rs_rank,
             int64_t ldd, int64_t m_rot, torch::Tensor status, int64_t bn, c10::optional<torch::Tensor> rmaps) {
  const c10::cuda::CUDAGuard g(a.device());
  TORCH_CHECK(a.size(1) == b.size(1), "gemm_rs: K mismatch");
  Operand A = classify(a, "a"), B = classify(b, "b");
  TORCH_CHECK(rptrs.is_cuda() && rptrs.scalar_type() == torch::kInt64, "gemm_rs: rptrs int64 cuda");
  LkGemmDesc d{};
  d.a = A.base; d.a_rows = A.rows; d.a_cols = A.cols; d.a_ld = A.ld; d.a_mn = A.mn;
  d.b = B.base; d.b_rows = B.rows; d.b_cols = B.cols; d.b_ld = B.ld; d.b_mn = B.mn;
  d.M = (int)a.size(0);
  d.N = (int)b.size(0);
  d.K = (int)a.size(1);
  TORCH_CHECK(d.M % rs_rows == 0 && d.M / rs_rows == rptrs.numel(), "gemm_rs: M must be world * rs_rows");
  TORCH_CHECK(ldd >= d.N && ldd % 8 == 0, "gemm_rs: ldd");
  d.ldd = ldd;
  d.alpha = 1.f;
  d.epi = LK_EPI_REMOTE;
  d.bn = (int)bn;
  need(status, "status", torch::kInt32);
  d.status = status.data_ptr<int>();
  d.comm_mode = 1;
  d.m_rot = (int)m_rot;
  d.rptrs = reinterpret_cast<void* const*>(rptrs.data_ptr());
  d.rs_rows = (int)rs_rows;
  d.rs_rank = (int)rs_rank;
  if (rmaps.has_value()) {
    TORCH_CHECK(rmaps->is_cuda() && rmaps->numel() == rptrs.numel() * 128 &&
                    reinterpret_cast<uintptr_t>(rmaps->data_ptr()) % 64 == 0,
                "gemm_rs: rmaps must be world x 128-byte tensor maps on the device");
    d.rmaps = rmaps->data_ptr();
  }
  check(lk_gemm(&d, stream()));
}

// K16: all-gather of A's rows from every rank's staging buffer (pointers in
// `src_ptrs`, int64 device tensor) into `a` on first use, fused with the GEMM.
void gemm_ag(torch::Tensor a, torch::Tensor b, torch::Tensor out, int64_t epi,
             c10::optional<torch::Tensor> h, torch::Tensor src_ptrs, int64_t src_ld, int64_t rows,
             int64_t rank, torch::Tensor count, int64_t m_rot, torch::Tensor status, int64_t bn) {
  const c10::cuda::CUDAGuard g(a.device());
  TORCH_CHECK(a.size(1) == b.size(1), "gemm_ag: K mismatch");
  Operand A = classify(a, "a"), B = classify(b, "b");
  TORCH_CHECK(!A.mn && a.stride(0) == A.ld, "gemm_ag: a must be row-major");
  TORCH_CHECK(src_ptrs.is_cuda() && src_ptrs.scalar_type() == torch::kInt64, "gemm_ag: src_ptrs");
  LkGemmDesc d{};
  d.a = A.base; d.a_rows = A.rows; d.a_cols = A.cols; d.a_ld = A.ld; d.a_mn = A.mn;
  d.b = B.base; d.b_rows = B.rows; d.b_cols = B.cols; d.b_ld = B.ld; d.b_mn = B.mn;
  d.M = (int)a.size(0);
  d.N = (int)b.size(0);
  d.K = (int)a.size(1);
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == torch::kBFloat16 && out.size(0) == d.M &&
                  out.size(1) == d.N && out.stride(1) == 1,
              "gemm_ag: out must be bf16 [M, N]");
  d.d = out.data_ptr();
  d.ldd = out.stride(0);
  if (h.has_value()) {
    need(*h, "h", torch::kBFloat16);
    TORCH_CHECK(h->size(0) == d.M && h->size(1) == d.N / 2 && h->stride(1) == 1, "gemm_ag: h shape");
    d.h = h->data_ptr();
    d.ldh = h->stride(0);
  }
  d.alpha = 1.f;
  d.epi = (int)epi;
  d.bn = (int)bn;
  need(status, "status", torch::kInt32);
  d.status = status.data_ptr<int>();
  need(count, "count", torch::kInt32);
  TORCH_CHECK(count.numel() >= d.M / 128, "gemm_ag: count too small");
  d.comm_mode = 2;
  d.m_rot = (int)m_rot;
  d.ag_src = reinterpret_cast<const void* const*>(src_ptrs.data_ptr());
  d.ag_ld_src = src_ld * 2;
  d.ag_rows = (int)rows;
  d.ag_rank = (int)rank;
  d.ag_world = (int)src_ptrs.numel();
  d.ag_count = count.data_ptr<int>();
  check(lk_gemm(&d, stream()));
}

// K17: ZeRO-3 group gather fused into the first GEMM that consumes it.  `b`
// is a view of `dst` (the local group buffer) at element `boff`.
void gemm_gather(torch::Tensor a, torch::Tensor b, torch::Tensor out, int64_t epi,
                 c10::optional<torch::Tensor> h, torch::Tensor src_ptrs, int64_t chunk, torch::Tensor dst,
                 int64_t boff, int64_t rank, torch::Tensor count, torch::Tensor status, int64_t bn) {
  const c10::cuda::CUDAGuard g(a.device());
  TORCH_CHECK(a.size(1) == b.size(1), "gemm_gather: K mismatch");
  Operand A = classify(a, "a"), B = classify(b, "b");
  TORCH_CHECK(!A.mn, "gemm_gather: A must be K-major");
  need_contig(dst, "dst", torch::kBFloat16);
  TORCH_CHECK(src_ptrs.is_cuda() && src_ptrs.scalar_type() == torch::kInt64, "gemm_gather: src_ptrs");
  LkGemmDesc d{};
  d.a = A.base; d.a_rows = A.rows; d.a_cols = A.cols; d.a_ld = A.ld; d.a_mn = A.mn;
  d.b = B.base; d.b_rows = B.rows; d.b_cols = B.cols; d.b_ld = B.ld; d.b_mn = B.mn;
  d.M = (int)a.size(0);
  d.N = (int)b.size(0);
  d.K = (int)a.size(1);
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == torch::kBFloat16 && out.size(0) == d.M &&
                  out.size(1) == d.N && out.stride(1) == 1,
              "gemm_gather: out must be bf16 [M, N]");
  d.d = out.data_ptr();
  d.ldd = out.stride(0);
  if (h.has_value()) {
    need(*h, "h", torch::kBFloat16);
    TORCH_CHECK(h->size(0) == d.M && h->size(1) == d.N / 2 && h->stride(1) == 1, "gemm_gather: h shape");
    d.h = h->data_ptr();
    d.ldh = h->stride(0);
  }
  d.alpha = 1.f;
  d.epi = (int)epi;
  d.bn = (int)bn;
  need(status, "status", torch::kInt32);
  d.status = status.data_ptr<int>();
  need(count, "count", torch::kInt32);
  TORCH_CHECK(count.numel() >= (d.N + 127) / 128, "gemm_gather: count too small");
  d.comm_mode = 3;
  d.ag_rank = (int)rank;
  d.ag_world = (int)src_ptrs.numel();
  d.gb_src = reinterpret_cast<const void* const*>(src_ptrs.data_ptr());
  d.gb_chunk = chunk;
  d.gb_len = dst.numel();
  d.gb_boff = boff;
  d.gb_dst = dst.data_ptr();
  d.gb_count = count.data_ptr<int>();
  check(lk_gemm(&d, stream()));
}

// K2: block-scaled fp8 GEMM and its quantisers.
void gemm_fp8(torch::Tensor a8, torch::Tensor sa, int64_t a_fmt, torch::Tensor b8, torch::Tensor sb,
              torch::Tensor out, c10::optional<torch::Tensor> resid, torch::Tensor status) {
  const c10::cuda::CUDAGuard g(a8.device());
  TORCH_CHECK(a8.is_cuda() && a8.scalar_type() == torch::kUInt8 && a8.dim() == 2 && a8.stride(1) == 1,
              "gemm_fp8: a8 must be a row-major uint8 (fp8 bits) matrix");
  TORCH_CHECK(b8.is_cuda() && b8.scalar_type() == torch::kUInt8 && b8.dim() == 2 && b8.stride(1) == 1,
              "gemm_fp8: b8 must be a row-major uint8 (fp8 bits) matrix");
  TORCH_CHECK(a8.size(1) == b8.size(1), "gemm_fp8: K mismatch");
  need_contig(sa, "sa", torch::kFloat32);
  need_contig(sb, "sb", torch::kFloat32);
  need(out, "out", torch::kBFloat16);
  LkGemmFp8Desc d{};
  d.a = a8.data_ptr();
  d.a_ld = a8.stride(0);
  d.b = b8.data_ptr();
  d.b_ld = b8.stride(0);
  d.M = (int)a8.size(0);
  d.N = (int)b8.size(0);
  d.K = (int)a8.size(1);
  d.a_fmt = (int)a_fmt;
  TORCH_CHECK(sa.numel() >= (int64_t)(d.K / 128) * d.M, "gemm_fp8: sa [K/128, M]");
  TORCH_CHECK(sb.numel() >= (int64_t)((d.N + 127) / 128) * (d.K / 128), "gemm_fp8: sb [N/128, K/128]");
  d.sa = sa.data_ptr<float>();
  d.sb = sb.data_ptr<float>();
  TORCH_CHECK(out.size(0) == d.M && out.size(1) == d.N && out.stride(1) == 1, "gemm_fp8: out [M, N]");
  d.d = out.data_ptr();
  d.ldd = out.stride(0);
  if (resid.has_value()) {
    need(*resid, "resid", torch::kBFloat16);
    TORCH_CHECK(resid->size(0) == d.M && resid->size(1) == d.N && resid->stride(1) == 1, "gemm_fp8: resid");
    d.r = resid->data_ptr();
    d.ldr = resid->stride(0);
  }
  need(status, "status", torch::kInt32);
  d.status = status.data_ptr<int>();
  check(lk_gemm_fp8(&d, stream()));
}

// K2 with a fused collective: mode "ag" (all-gather of A's fp8 rows + scales into
// a8 / sa) or "rs" (reduce-scatter epilogue into the owners' receive buffers).
void gemm_fp8_comm(torch::Tensor a8, torch::Tensor sa, int64_t a_fmt, torch::Tensor b8, torch::Tensor sb,
                   c10::optional<torch::Tensor> out, torch::Tensor status, int64_t rank, int64_t world,
                   c10::optional<torch::Tensor> ag_rows, c10::optional<torch::Tensor> ag_scales,
                   int64_t rows_per_rank, c10::optional<torch::Tensor> count, c10::optional<torch::Tensor> rptrs,
                   int64_t rs_rows, int64_t ldd) {
  const c10::cuda::CUDAGuard g(a8.device());
  TORCH_CHECK(a8.is_cuda() && a8.scalar_type() == torch::kUInt8 && a8.dim() == 2 && a8.stride(1) == 1, "a8");
  TORCH_CHECK(b8.is_cuda() && b8.scalar_type() == torch::kUInt8 && b8.dim() == 2 && b8.stride(1) == 1, "b8");
  TORCH_CHECK(a8.size(1) == b8.size(1), "gemm_fp8_comm: K mismatch");
  need_contig(sa, "sa", torch::kFloat32);
  need_contig(sb, "sb", torch::kFloat32);
  LkGemmFp8Desc d{};
  d.a = a8.data_ptr();
  d.a_ld = a8.stride(0);
  d.b = b8.data_ptr();
  d.b_ld = b8.stride(0);
  d.M = (int)a8.size(0);
  d.N = (int)b8.size(0);
  d.K = (int)a8.size(1);
  d.a_fmt = (int)a_fmt;
  d.sa = sa.data_ptr<float>();
  d.sb = sb.data_ptr<float>();
  need(status, "status", torch::kInt32);
  d.status = status.data_ptr<int>();
  d.rank = (int)rank;
  d.world = (int)world;
  if (ag_rows.has_value()) {
    TORCH_CHECK(ag_scales.has_value() && count.has_value() && out.has_value(), "gemm_fp8_comm ag: missing args");
    d.ag_rows = reinterpret_cast<const void* const*>(ag_rows->data_ptr());
    d.ag_scales = reinterpret_cast<const float* const*>(ag_scales->data_ptr());
    d.ag_rows_per_rank = (int)rows_per_rank;
    d.ag_count = count->data_ptr<int>();
  }
  if (out.has_value()) {
    need(*out, "out", torch::kBFloat16);
    TORCH_CHECK(out->size(0) == d.M && out->size(1) == d.N && out->stride(1) == 1, "gemm_fp8_comm: out");
    d.d = out->data_ptr();
    d.ldd = out->stride(0);
  }
  if (rptrs.has_value()) {
    d.rptrs = reinterpret_cast<void* const*>(rptrs->data_ptr());
    d.rs_rows = (int)rs_rows;
    d.ldd = ldd;
  }
  check(lk_gemm_fp8(&d, stream()));
}

void dequant_1x128(torch::Tensor q, int64_t fmt, torch::Tensor scale, torch::Tensor x) {
  const c10::cuda::CUDAGuard g(q.device());
  TORCH_CHECK(q.is_contiguous() && q.scalar_type() == torch::kUInt8 && q.dim() == 2, "dequant_1x128: q");
  need_contig(scale, "scale", torch::kFloat32);
  need(x, "x", torch::kBFloat16);
  TORCH_CHECK(x.size(0) == q.size(0) && x.size(1) == q.size(1) && x.stride(1) == 1, "dequant_1x128: x");
  check(lk_dequant_1x128(q.data_ptr(), (int)q.size(0), (int)q.size(1), (int)fmt, scale.data_ptr<float>(),
                         x.data_ptr(), x.stride(0), stream()));
}

void quant_1x128(torch::Tensor x, int64_t fmt, torch::Tensor q, torch::Tensor scale) {
  const c10::cuda::CUDAGuard g(x.device());
  need(x, "x", torch::kBFloat16);
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1, "quant_1x128: x row-major");
  TORCH_CHECK(q.scalar_type() == torch::kUInt8 && q.stride(1) == 1 && q.size(0) == x.size(0) &&
                  q.size(1) == x.size(1), "quant_1x128: q");
  need_contig(scale, "scale", torch::kFloat32);
  TORCH_CHECK(scale.numel() >= x.size(0) * (x.size(1) / 128), "quant_1x128: scale");
  check(lk_quant_1x128(x.data_ptr(), x.stride(0), (int)x.size(0), (int)x.size(1), (int)fmt, q.data_ptr(),
                       q.stride(0), scale.data_ptr<float>(), stream()));
}

void quant_128x128(torch::Tensor w, torch::Tensor q, c10::optional<torch::Tensor> qt, torch::Tensor scale) {
  const c10::cuda::CUDAGuard g(w.device());
  need(w, "w", torch::kBFloat16);
  TORCH_CHECK(w.dim() == 2 && w.stride(1) == 1, "quant_128x128: w row-major");
  TORCH_CHECK(q.is_contiguous() && q.scalar_type() == torch::kUInt8 && q.numel() == w.numel(), "quant_128x128: q");
  if (qt.has_value())
    TORCH_CHECK(qt->is_contiguous() && qt->scalar_type() == torch::kUInt8 && qt->numel() == w.numel(),
                "quant_128x128: qt");
  need_contig(scale, "scale", torch::kFloat32);
  TORCH_CHECK(scale.numel() >= ((w.size(0) + 127) / 128) * (w.size(1) / 128), "quant_128x128: scale");
  check(lk_quant_128x128(w.data_ptr(), w.stride(0), (int)w.size(0), (int)w.size(1), q.data_ptr(),
                         qt.has_value() ? qt->data_ptr() : nullptr, scale.data_ptr<float>(), stream()));
}

// K2, MX form: hardware block-scaled fp8 GEMM (UE8M0 SF tiles) and its quantisers.
static void mx_operand(const torch::Tensor& t, const char* what) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == torch::kUInt8 && t.dim() == 2 && t.stride(1) == 1, what,
              " must be a row-major uint8 (fp8 bits) matrix");
}

static int64_t mx_sf_bytes(int64_t row_tiles, int64_t K) { return row_tiles * (K / 128) * 512; }

void gemm_mxf8(torch::Tensor a8, torch::Tensor sfa, int64_t a_fmt, torch::Tensor b8, torch::Tensor sfb,
               int64_t b_fmt, c10::optional<torch::Tensor> out, c10::optional<torch::Tensor> resid,
               torch::Tensor status, int64_t rank, int64_t world, c10::optional<torch::Tensor> ag_rows,
               c10::optional<torch::Tensor> ag_sf, int64_t rows_per_rank, c10::optional<torch::Tensor> count,
               c10::optional<torch::Tensor> rptrs, int64_t rs_rows, int64_t ldd) {
  const c10::cuda::CUDAGuard g(a8.device());
  mx_operand(a8, "gemm_mxf8: a8");
  mx_operand(b8, "gemm_mxf8: b8");
  TORCH_CHECK(a8.size(1) == b8.size(1), "gemm_mxf8: K mismatch");
  TORCH_CHECK(sfa.is_cuda() && sfa.is_contiguous() && sfa.scalar_type() == torch::kUInt8, "gemm_mxf8: sfa uint8");
  TORCH_CHECK(sfb.is_cuda() && sfb.is_contiguous() && sfb.scalar_type() == torch::kUInt8, "gemm_mxf8: sfb uint8");
  LkGemmMxf8Desc d{};
  d.a = a8.data_ptr();
  d.a_ld = a8.stride(0);
  d.b = b8.data_ptr();
  d.b_ld = b8.stride(0);
  d.M = (int)a8.size(0);
  d.N = (int)b8.size(0);
  d.K = (int)a8.size(1);
  d.a_fmt = (int)a_fmt;
  d.b_fmt = (int)b_fmt;
  TORCH_CHECK(sfa.numel() >= mx_sf_bytes((d.M + 127) / 128, d.K), "gemm_mxf8: sfa holds ceil(M/128) row tiles");
  TORCH_CHECK(sfb.numel() >= mx_sf_bytes(2 * ((d.N + 255) / 256), d.K),
              "gemm_mxf8: sfb holds 2 ceil(N/256) row tiles");
  d.sfa = sfa.data_ptr();
  d.sfb = sfb.data_ptr();
  need(status, "status", torch::kInt32);
  d.status = status.data_ptr<int>();
  d.rank = (int)rank;
  d.world = (int)world;
  if (out.has_value()) {
    need(*out, "out", torch::kBFloat16);
    TORCH_CHECK(out->size(0) == d.M && out->size(1) == d.N && out->stride(1) == 1, "gemm_mxf8: out [M, N]");
    d.d = out->data_ptr();
    d.ldd = out->stride(0);
  }
  if (resid.has_value()) {
    need(*resid, "resid", torch::kBFloat16);
    TORCH_CHECK(resid->size(0) == d.M && resid->size(1) == d.N && resid->stride(1) == 1, "gemm_mxf8: resid");
    d.r = resid->data_ptr();
    d.ldr = resid->stride(0);
  }
  if (ag_rows.has_value()) {
    TORCH_CHECK(ag_sf.has_value() && count.has_value() && out.has_value(), "gemm_mxf8 ag: missing args");
    d.ag_rows = reinterpret_cast<const void* const*>(ag_rows->data_ptr());
    d.ag_sf = reinterpret_cast<const void* const*>(ag_sf->data_ptr());
    d.ag_rows_per_rank = (int)rows_per_rank;
    d.ag_count = count->data_ptr<int>();
  }
  if (rptrs.has_value()) {
    d.rptrs = reinterpret_cast<void* const*>(rptrs->data_ptr());
    d.rs_rows = (int)rs_rows;
    d.ldd = ldd;
  } else {
    TORCH_CHECK(out.has_value(), "gemm_mxf8: out required");
  }
  check(lk_gemm_mxf8(&d, stream()));
}

void quant_mx_rows(torch::Tensor x, int64_t fmt, torch::Tensor q, torch::Tensor sf, int64_t rows_pad) {
  const c10::cuda::CUDAGuard g(x.device());
  need(x, "x", torch::kBFloat16);
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1, "quant_mx_rows: x row-major");
  TORCH_CHECK(q.scalar_type() == torch::kUInt8 && q.stride(1) == 1 && q.size(0) == x.size(0) &&
                  q.size(1) == x.size(1), "quant_mx_rows: q");
  TORCH_CHECK(sf.is_contiguous() && sf.scalar_type() == torch::kUInt8 &&
                  sf.numel() >= mx_sf_bytes(rows_pad / 128, x.size(1)), "quant_mx_rows: sf");
  check(lk_quant_mx_rows(x.data_ptr(), x.stride(0), (int)x.size(0), (int)rows_pad, (int)x.size(1), (int)fmt,
                         q.data_ptr(), q.stride(0), sf.data_ptr(), stream()));
}

void quant_mx_128x128(torch::Tensor w, torch::Tensor q, torch::Tensor sf, torch::Tensor scale,
                      c10::optional<torch::Tensor> qt, c10::optional<torch::Tensor> sft) {
  const c10::cuda::CUDAGuard g(w.device());
  need(w, "w", torch::kBFloat16);
  TORCH_CHECK(w.dim() == 2 && w.stride(1) == 1, "quant_mx_128x128: w row-major");
  const int64_t N = w.size(0), K = w.size(1);
  TORCH_CHECK(q.is_contiguous() && q.scalar_type() == torch::kUInt8 && q.numel() == w.numel(), "quant_mx_128x128: q");
  TORCH_CHECK(sf.is_contiguous() && sf.scalar_type() == torch::kUInt8 && sf.numel() >= mx_sf_bytes((N + 127) / 128, K),
              "quant_mx_128x128: sf");
  need_contig(scale, "scale", torch::kFloat32);
  TORCH_CHECK(scale.numel() >= ((N + 127) / 128) * (K / 128), "quant_mx_128x128: scale");
  TORCH_CHECK(qt.has_value() == sft.has_value(), "quant_mx_128x128: qt and sft together");
  if (qt.has_value()) {
    TORCH_CHECK(qt->is_contiguous() && qt->scalar_type() == torch::kUInt8 && qt->numel() == w.numel(),
                "quant_mx_128x128: qt");
    TORCH_CHECK(sft->is_contiguous() && sft->scalar_type() == torch::kUInt8 &&
                    sft->numel() >= mx_sf_bytes(K / 128, N), "quant_mx_128x128: sft");
  }
  check(lk_quant_mx_128x128(w.data_ptr(), w.stride(0), (int)N, (int)K, q.data_ptr(), sf.data_ptr(),
                            scale.data_ptr<float>(), qt.has_value() ? qt->data_ptr() : nullptr,
                            sft.has_value() ? sft->data_ptr() : nullptr, stream()));
}

void dequant_mx_rows(torch::Tensor q, int64_t fmt, torch::Tensor sf, torch::Tensor x) {
  const c10::cuda::CUDAGuard g(q.device());
  TORCH_CHECK(q.is_contiguous() && q.scalar_type() == torch::kUInt8 && q.dim() == 2, "dequant_mx_rows: q");
  TORCH_CHECK(sf.is_contiguous() && sf.scalar_type() == torch::kUInt8 &&
                  sf.numel() >= mx_sf_bytes((q.size(0) + 127) / 128, q.size(1)), "dequant_mx_rows: sf");
  need(x, "x", torch::kBFloat16);
  TORCH_CHECK(x.size(0) == q.size(0) && x.size(1) == q.size(1) && x.stride(1) == 1, "dequant_mx_rows: x");
  check(lk_dequant_mx_rows(q.data_ptr(), (int)q.size(0), (int)q.size(1), (int)fmt, sf.data_ptr(), x.data_ptr(),
                           x.stride(0), stream()));
}

// K14 decode form: weight-streaming dequant GEMM (tcgen05), M <= 256.
void dq_gemm(torch::Tensor x, torch::Tensor q, torch::Tensor scale, c10::optional<torch::Tensor> zero, int64_t fmt,
             int64_t N, int64_t K, int64_t group, torch::Tensor y, c10::optional<torch::Tensor> resid,
             c10::optional<torch::Tensor> partial, int64_t splits, torch::Tensor status,
             c10::optional<torch::Tensor> counters) {
  const c10::cuda::CUDAGuard g(x.device());
  need(x, "x", torch::kBFloat16);
  need(y, "y", torch::kBFloat16);
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1 && x.size(1) == K, "dq_gemm: x [M, K] row-major");
  TORCH_CHECK(y.dim() == 2 && y.stride(1) == 1 && y.size(0) == x.size(0) && y.size(1) == N, "dq_gemm: y [M, N]");
  TORCH_CHECK(q.is_cuda() && q.is_contiguous(), "dq_gemm: q contiguous");
  need_contig(scale, "scale", torch::kFloat32);
  LkDqGemmDesc d{};
  d.fmt = (int)fmt;
  d.x = x.data_ptr();
  d.ldx = x.stride(0);
  d.M = (int)x.size(0);
  d.q = q.data_ptr();
  d.scale = scale.data_ptr<float>();
  d.zero = optp<float>(zero);
  d.N = (int)N;
  d.K = (int)K;
  d.group = (int)group;
  d.y = y.data_ptr();
  d.ldy = y.stride(0);
  if (resid.has_value()) {
    need(*resid, "resid", torch::kBFloat16);
    TORCH_CHECK(resid->size(0) == d.M && resid->size(1) == N && resid->stride(1) == 1, "dq_gemm: resid");
    d.r = resid->data_ptr();
    d.ldr = resid->stride(0);
  }
  d.splits = (int)splits;
  if (partial.has_value()) {
    need_contig(*partial, "partial", torch::kFloat32);
    TORCH_CHECK(partial->numel() >= (int64_t)std::max<int64_t>(splits, 1) * d.M * N, "dq_gemm: partial size");
    d.partial = partial->data_ptr<float>();
  }
  if (counters.has_value()) {
    need_contig(*counters, "counters", torch::kInt32);
    TORCH_CHECK(counters->numel() >= LK_DQ_COUNTERS, "dq_gemm: counters need LK_DQ_COUNTERS entries");
    d.counters = counters->data_ptr<int>();
  }
  need(status, "status", torch::kInt32);
  d.status = status.data_ptr<int>();
  check(lk_dq_gemm(&d, stream()));
}

int64_t dq_gemm_splits(int64_t M, int64_t N, int64_t K) { return lk_dq_gemm_splits((int)M, (int)N, (int)K); }

// K18 owner side: sum of the received slots (+ residual, + RMSNorm).
void rs_sum(torch::Tensor recv, int64_t world, torch::Tensor out, c10::optional<torch::Tensor> resid,
            c10::optional<torch::Tensor> gamma, c10::optional<torch::Tensor> y,
            c10::optional<torch::Tensor> rstd, double eps, int64_t src_mode,
            c10::optional<torch::Tensor> peers, int64_t mc) {
  const c10::cuda::CUDAGuard g(recv.device());
  need(recv, "recv", torch::kBFloat16);
  need(out, "out", torch::kBFloat16);
  TORCH_CHECK(recv.dim() == 2 && recv.stride(1) == 1 && out.stride(1) == 1, "rs_sum: row-major");
  LkRsSumDesc d{};
  d.recv = recv.data_ptr();
  d.ld_recv = recv.stride(0);
  d.world = (int)world;
  d.rows = (int)out.size(0);
  d.cols = (int)out.size(1);
  TORCH_CHECK(recv.size(0) >= (src_mode == 0 ? world : 1) * d.rows && recv.size(1) >= d.cols, "rs_sum: recv shape");
  d.src_mode = (int)src_mode;
  if (src_mode == 1) {
    TORCH_CHECK(peers.has_value() && peers->is_cuda() && peers->scalar_type() == torch::kInt64 &&
                    peers->numel() == world, "rs_sum: peers must be an int64 device array of world pointers");
    d.peers = reinterpret_cast<const void* const*>(peers->data_ptr());
  } else if (src_mode == 2) {
    TORCH_CHECK(mc != 0, "rs_sum: multicast address needed");
    d.mc = reinterpret_cast<const void*>(mc);
  }
  d.out = out.data_ptr();
  d.ld_out = out.stride(0);
  if (resid.has_value()) {
    need(*resid, "resid", torch::kBFloat16);
    TORCH_CHECK(resid->size(0) == d.rows && resid->size(1) == d.cols && resid->stride(1) == 1, "rs_sum: resid");
    d.resid = resid->data_ptr();
    d.ld_resid = resid->stride(0);
  }
  if (gamma.has_value()) {
    TORCH_CHECK(y.has_value(), "rs_sum: y needed with gamma");
    need_contig(*gamma, "gamma", torch::kBFloat16);
    need(*y, "y", torch::kBFloat16);
    TORCH_CHECK(y->size(0) == d.rows && y->size(1) == d.cols && y->stride(1) == 1, "rs_sum: y shape");
    d.gamma = gamma->data_ptr();
    d.y = y->data_ptr();
    d.ld_y = y->stride(0);
    d.rstd = optp<float>(rstd);
    d.eps = (float)eps;
  }
  check(lk_rs_sum(&d, stream()));
}

// Vocabulary-parallel cross-entropy (phase 1: statistics, phase 2: finish).
void cross_entropy_vp(torch::Tensor logits, torch::Tensor targets, torch::Tensor loss_acc,
                      c10::optional<torch::Tensor> scale, double scale_mul, double smoothing,
                      double zloss, int64_t ignore_index, bool write_grad, int64_t v0,
                      int64_t v_total, torch::Tensor stats, torch::Tensor peer_stats, int64_t phase) {
  const c10::cuda::CUDAGuard g(logits.device());
  need(logits, "logits", torch::kBFloat16);
  TORCH_CHECK(logits.dim() == 2 && logits.stride(1) == 1, "cross_entropy_vp: logits row-major");
  need_contig(targets, "targets", torch::kInt64);
  LkCeVpDesc d{};
  d.ce.logits = logits.data_ptr();
  d.ce.ld = logits.stride(0);
  d.ce.targets = targets.data_ptr<int64_t>();
  d.ce.T = (int)logits.size(0);
  d.ce.V = (int)logits.size(1);
  TORCH_CHECK(targets.numel() == d.ce.T, "cross_entropy_vp: targets");
  d.ce.loss_acc = loss_acc.data_ptr<float>();
  d.ce.scale_ptr = optp<const float>(scale);
  d.ce.scale_mul = (float)scale_mul;
  d.ce.smoothing = (float)smoothing;
  d.ce.zloss = (float)zloss;
  d.ce.ignore_index = ignore_index;
  d.ce.write_grad = write_grad ? 1 : 0;
  d.v0 = v0;
  d.V_total = v_total;
  need(stats, "stats", torch::kFloat32);
  TORCH_CHECK(stats.numel() >= 4 * d.ce.T, "cross_entropy_vp: stats [T, 4]");
  d.stats = stats.data_ptr<float>();
  TORCH_CHECK(peer_stats.is_cuda() && peer_stats.scalar_type() == torch::kInt64, "peer_stats int64");
  d.peer_stats = reinterpret_cast<const float* const*>(peer_stats.data_ptr());
  d.world = (int)peer_stats.numel();
  d.phase = (int)phase;
  check(lk_cross_entropy_vp(&d, stream()));
}

// ------------------------------------------------------ GELU, LayerNorm
void cast_f32_bf16(torch::Tensor x, torch::Tensor y) {
  const c10::cuda::CUDAGuard g(x.device());
  need_contig(x, "x", torch::kFloat32);
  need_contig(y, "y", torch::kBFloat16);
  TORCH_CHECK(x.numel() == y.numel(), "cast_f32_bf16: sizes");
  check(lk_cast_f32_bf16(x.data_ptr<float>(), y.data_ptr(), x.numel(), stream()));
}

void gelu_fwd(torch::Tensor x, torch::Tensor y) {
  const c10::cuda::CUDAGuard g(x.device());
  need_contig(x, "x", torch::kBFloat16);
  need_contig(y, "y", torch::kBFloat16);
  TORCH_CHECK(x.numel() == y.numel(), "gelu: sizes");
  check(lk_gelu_fwd(x.data_ptr(), y.data_ptr(), x.numel(), stream()));
}

void gelu_bwd(torch::Tensor x, torch::Tensor dy, torch::Tensor dx) {
  const c10::cuda::CUDAGuard g(x.device());
  need_contig(x, "x", torch::kBFloat16);
  need_contig(dy, "dy", torch::kBFloat16);
  need_contig(dx, "dx", torch::kBFloat16);
  TORCH_CHECK(x.numel() == dy.numel() && x.numel() == dx.numel(), "gelu: sizes");
  check(lk_gelu_bwd(x.data_ptr(), dy.data_ptr(), dx.data_ptr(), x.numel(), stream()));
}

void dropout(torch::Tensor x, torch::Tensor y, double p, int64_t seed) {
  const c10::cuda::CUDAGuard g(x.device());
  need_contig(x, "x", torch::kBFloat16);
  need_contig(y, "y", torch::kBFloat16);
  TORCH_CHECK(x.numel() == y.numel(), "dropout: sizes");
  check(lk_dropout(x.data_ptr(), y.data_ptr(), x.numel(), (float)p, (uint64_t)seed, stream()));
}

void layernorm_fwd(torch::Tensor x, torch::Tensor gamma, torch::Tensor beta, torch::Tensor y, torch::Tensor mean,
                   torch::Tensor rstd, double eps) {
  const c10::cuda::CUDAGuard g(x.device());
  need_contig(x, "x", torch::kBFloat16);
  need_contig(gamma, "gamma", torch::kBFloat16);
  need_contig(beta, "beta", torch::kBFloat16);
  need_contig(y, "y", torch::kBFloat16);
  need_contig(mean, "mean", torch::kFloat32);
  need_contig(rstd, "rstd", torch::kFloat32);
  const int D = (int)x.size(-1), M = (int)(x.numel() / D);
  TORCH_CHECK(gamma.numel() == D && beta.numel() == D && mean.numel() >= M && rstd.numel() >= M, "layernorm: shapes");
  check(lk_layernorm_fwd(x.data_ptr(), gamma.data_ptr(), beta.data_ptr(), y.data_ptr(), mean.data_ptr<float>(),
                         rstd.data_ptr<float>(), M, D, (float)eps, stream()));
}

void layernorm_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor gamma, torch::Tensor mean, torch::Tensor rstd,
                   torch::Tensor dx, torch::Tensor dgamma, torch::Tensor dbeta) {
  const c10::cuda::CUDAGuard g(x.device());
  need_contig(dy, "dy", torch::kBFloat16);
  need_contig(x, "x", torch::kBFloat16);
  need_contig(gamma, "gamma", torch::kBFloat16);
  need_contig(dx, "dx", torch::kBFloat16);
  need_contig(dgamma, "dgamma", torch::kFloat32);
  need_contig(dbeta, "dbeta", torch::kFloat32);
  const int D = (int)x.size(-1), M = (int)(x.numel() / D);
  check(lk_layernorm_bwd(dy.data_ptr(), x.data_ptr(), gamma.data_ptr(), mean.data_ptr<float>(),
                         rstd.data_ptr<float>(), dx.data_ptr(), dgamma.data_ptr<float>(), dbeta.data_ptr<float>(),
                         M, D, stream()));
}

// ------------------------------------------------------------- RMSNorm
void rmsnorm_fwd(torch::Tensor x, c10::optional<torch::Tensor> res, torch::Tensor gamma,
                 torch::Tensor y, c10::optional<torch::Tensor> h_out,
                 c10::optional<torch::Tensor> rstd, double eps) {
  const c10::cuda::CUDAGuard g(x.device());
  need_contig(x, "x", torch::kBFloat16);
  need_contig(gamma, "gamma", torch::kBFloat16);
  need_contig(y, "y", torch::kBFloat16);
  LkNormFwdDesc d{};
  d.D = (int)x.size(-1);
  d.M = (int)(x.numel() / d.D);
  d.x = x.data_ptr();
  d.res = optp(res);
  d.gamma = gamma.data_ptr();
  d.y = y.data_ptr();
  d.h_out = optp(h_out);
  d.rstd = optp<float>(rstd);
  d.eps = (float)eps;
  check(lk_rmsnorm_fwd(&d, stream()));
}

void rmsnorm_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor gamma, torch::Tensor rstd,
                 c10::optional<torch::Tensor> dres, torch::Tensor dx, torch::Tensor dgamma,
                 torch::Tensor partial, bool accumulate) {
  const c10::cuda::CUDAGuard g(x.device());
  need_contig(dy, "dy", torch::kBFloat16);
  need_contig(x, "x", torch::kBFloat16);
  need_contig(dx, "dx", torch::kBFloat16);
  need_contig(rstd, "rstd", torch::kFloat32);
  const bool g16 = dgamma.scalar_type() == torch::kBFloat16;
  need_contig(dgamma, "dgamma", g16 ? torch::kBFloat16 : torch::kFloat32);
  TORCH_CHECK(!g16 || !accumulate, "rmsnorm_bwd: a bf16 dgamma is stored, not accumulated");
  need_contig(partial, "partial", torch::kFloat32);
  LkNormBwdDesc d{};
  d.dgamma_bf16 = g16 ? 1 : 0;
  d.D = (int)x.size(-1);
  d.M = (int)(x.numel() / d.D);
  d.dy = dy.data_ptr();
  d.x = x.data_ptr();
  d.gamma = gamma.data_ptr();
  d.rstd = rstd.data_ptr<float>();
  d.dres = optp(dres);
  d.dx = dx.data_ptr();
  d.dgamma = reinterpret_cast<float*>(dgamma.data_ptr());
  d.partial = partial.data_ptr<float>();
  d.partial_rows = (int)(partial.numel() / d.D);
  d.accumulate = accumulate ? 1 : 0;
  check(lk_rmsnorm_bwd(&d, stream()));
}

int64_t rmsnorm_bwd_partial_rows(int64_t M) { return lk_rmsnorm_bwd_partial_rows((int)M); }

// --------------------------------------------------------- RoPE / SwiGLU / emb
void rope(torch::Tensor x, int64_t col0, int64_t nheads, int64_t Dh, torch::Tensor table,
          c10::optional<torch::Tensor> pos, int64_t seq_len, int64_t pos_offset, bool inverse) {
  const c10::cuda::CUDAGuard g(x.device());
  need(x, "x", torch::kBFloat16);
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1, "rope: x must be a row-major 2-D view");
  need_contig(table, "table", torch::kFloat32);
  LkRopeDesc d{};
  d.x = x.data_ptr();
  d.ld = x.stride(0);
  d.T = (int)x.size(0);
  d.col0 = (int)col0;
  d.nheads = (int)nheads;
  d.Dh = (int)Dh;
  d.table = table.data_ptr();
  if (pos.has_value()) need_contig(*pos, "pos", torch::kInt32);
  d.pos = optp<int>(pos);
  d.seq_len = (int)seq_len;
  d.pos_offset = (int)pos_offset;
  d.inverse = inverse ? 1 : 0;
  TORCH_CHECK(col0 + nheads * Dh <= x.size(1), "rope: heads exceed the row");
  check(lk_rope(&d, stream()));
}

void swiglu_fwd(torch::Tensor gu, torch::Tensor h) {
  const c10::cuda::CUDAGuard g(gu.device());
  need_contig(gu, "gu", torch::kBFloat16);
  need_contig(h, "h", torch::kBFloat16);
  const int F = (int)h.size(-1);
  check(lk_swiglu_fwd(gu.data_ptr(), h.data_ptr(), (int)(h.numel() / F), F, stream()));
}

void swiglu_bwd(torch::Tensor gu, torch::Tensor dh, torch::Tensor dgu) {
  const c10::cuda::CUDAGuard g(gu.device());
  need_contig(gu, "gu", torch::kBFloat16);
  need_contig(dh, "dh", torch::kBFloat16);
  need_contig(dgu, "dgu", torch::kBFloat16);
  const int F = (int)dh.size(-1);
  check(lk_swiglu_bwd(gu.data_ptr(), dh.data_ptr(), dgu.data_ptr(), (int)(dh.numel() / F), F, stream()));
}

void embedding_fwd(torch::Tensor ids, torch::Tensor W, torch::Tensor out, torch::Tensor status) {
  const c10::cuda::CUDAGuard g(W.device());
  need_contig(ids, "ids", torch::kInt64);
  need_contig(W, "W", torch::kBFloat16);
  need_contig(out, "out", torch::kBFloat16);
  check(lk_embedding_fwd(ids.data_ptr<int64_t>(), W.data_ptr(), out.data_ptr(), (int)ids.numel(),
                         (int)W.size(1), (int)W.size(0), status.data_ptr<int>(), stream()));
}

void embedding_bwd(torch::Tensor ids, torch::Tensor dy, torch::Tensor dW) {
  const c10::cuda::CUDAGuard g(dW.device());
  need_contig(ids, "ids", torch::kInt64);
  need_contig(dy, "dy", torch::kBFloat16);
  need_contig(dW, "dW", torch::kFloat32);
  check(lk_embedding_bwd(ids.data_ptr<int64_t>(), dy.data_ptr(), dW.data_ptr<float>(),
                         (int)ids.numel(), (int)dW.size(1), (int)dW.size(0), stream()));
}

// ----------------------------------------------------------- cross-entropy
void cross_entropy(torch::Tensor logits, torch::Tensor targets, torch::Tensor loss_acc,
                   c10::optional<torch::Tensor> row_loss, c10::optional<torch::Tensor> scale,
                   double scale_mul, double smoothing, double zloss, int64_t ignore_index,
                   bool write_grad) {
  const c10::cuda::CUDAGuard g(logits.device());
  need(logits, "logits", torch::kBFloat16);
  TORCH_CHECK(logits.dim() == 2 && logits.stride(1) == 1, "cross_entropy: logits must be row-major 2-D");
  need_contig(targets, "targets", torch::kInt64);
  need_contig(loss_acc, "loss_acc", torch::kFloat32);
  LkCeDesc d{};
  d.logits = logits.data_ptr();
  d.ld = logits.stride(0);
  d.targets = targets.data_ptr<int64_t>();
  d.T = (int)logits.size(0);
  d.V = (int)logits.size(1);
  d.loss_acc = loss_acc.data_ptr<float>();
  d.row_loss = optp<float>(row_loss);
  d.scale_ptr = optp<float>(scale);
  d.scale_mul = (float)scale_mul;
  d.smoothing = (float)smoothing;
  d.zloss = (float)zloss;
  d.ignore_index = ignore_index;
  d.write_grad = write_grad ? 1 : 0;
  check(lk_cross_entropy(&d, stream()));
}

// ------------------------------------------------------------ optimizer
void adamw(torch::Tensor p32, torch::Tensor grad, torch::Tensor m, torch::Tensor v,
           c10::optional<torch::Tensor> p16, c10::optional<torch::Tensor> ema,
           torch::Tensor chunks, torch::Tensor state, double beta1, double beta2, double eps,
           double wd, double ema_decay, bool zero_grad, c10::optional<torch::Tensor> p16_peers) {
  const c10::cuda::CUDAGuard g(p32.device());
  need_contig(p32, "p32", torch::kFloat32);
  need_contig(grad, "grad", torch::kFloat32);
  need_contig(m, "m", torch::kFloat32);
  need_contig(v, "v", torch::kFloat32);
  need_contig(chunks, "chunks", torch::kInt32);
  need_contig(state, "state", torch::kFloat32);
  LkAdamWDesc d{};
  d.p32 = p32.data_ptr<float>();
  d.g = grad.data_ptr<float>();
  d.m = m.data_ptr<float>();
  d.v = v.data_ptr<float>();
  d.p16 = optp(p16);
  d.ema = optp<float>(ema);
  d.chunks = chunks.data_ptr<int>();
  d.nchunks = (int)(chunks.numel() / 4);
  d.state = state.data_ptr<float>();
  d.beta1 = (float)beta1;
  d.beta2 = (float)beta2;
  d.eps = (float)eps;
  d.wd = (float)wd;
  d.ema_decay = (float)ema_decay;
  d.zero_grad = zero_grad ? 1 : 0;
  if (p16_peers.has_value()) {
    TORCH_CHECK(p16_peers->is_cuda() && p16_peers->scalar_type() == torch::kInt64, "adamw: p16_peers");
    d.p16_peers = reinterpret_cast<void* const*>(p16_peers->data_ptr());
    d.world = (int)p16_peers->numel();
  }
  check(lk_adamw(&d, stream()));
}

void grad_norm_partials(torch::Tensor grad, torch::Tensor partial) {
  const c10::cuda::CUDAGuard g(grad.device());
  need_contig(grad, "grad", torch::kFloat32);
  need_contig(partial, "partial", torch::kFloat32);
  check(lk_grad_norm_partials(grad.data_ptr<float>(), grad.numel(), partial.data_ptr<float>(),
                              (int)partial.numel(), stream()));
}

void optimizer_finalize(torch::Tensor partial, torch::Tensor state, double max_norm, bool dynamic,
                        double growth, double backoff, int64_t growth_interval, double min_scale) {
  const c10::cuda::CUDAGuard g(state.device());
  need_contig(partial, "partial", torch::kFloat32);
  need_contig(state, "state", torch::kFloat32);
  check(lk_optimizer_finalize(partial.data_ptr<float>(), (int)partial.numel(), state.data_ptr<float>(),
                              (float)max_norm, dynamic ? 1 : 0, (float)growth, (float)backoff,
                              (int)growth_interval, (float)min_scale, stream()));
}

// ------------------------------------------------------------- attention
void attention_fwd(torch::Tensor qkv, torch::Tensor o, torch::Tensor lse, int64_t B, int64_t S,
                   int64_t Hq, int64_t Hkv, int64_t Dh, bool causal, int64_t window, double scale,
                   torch::Tensor status, c10::optional<torch::Tensor> kv, int64_t q_off) {
  const c10::cuda::CUDAGuard g(qkv.device());
  need(qkv, "qkv", torch::kBFloat16);
  need(o, "o", torch::kBFloat16);
  need_contig(lse, "lse", torch::kFloat32);
  const int64_t qcols = kv.has_value() ? Hq * Dh : (Hq + 2 * Hkv) * Dh;
  TORCH_CHECK(qkv.dim() == 2 && qkv.stride(1) == 1 && qkv.size(0) == B * S && qkv.size(1) >= qcols,
              "attention: bad qkv shape");
  TORCH_CHECK(o.dim() == 2 && o.stride(1) == 1 && o.size(0) == B * S && o.size(1) >= Hq * Dh,
              "attention: bad o shape");
  TORCH_CHECK(lse.numel() >= B * Hq * S, "attention: lse too small");
  LkAttnDesc d{};
  d.qkv = qkv.data_ptr();
  d.ld_qkv = qkv.stride(0);
  d.o = o.data_ptr();
  d.ld_o = o.stride(0);
  d.lse = lse.data_ptr<float>();
  d.B = (int)B; d.S = (int)S; d.Hq = (int)Hq; d.Hkv = (int)Hkv; d.Dh = (int)Dh;
  d.causal = causal ? 1 : 0;
  d.window = (int)window;
  d.scale = (float)scale;
  d.status = status.data_ptr<int>();
  if (kv.has_value()) {
    need(*kv, "kv", torch::kBFloat16);
    TORCH_CHECK(kv->dim() == 2 && kv->stride(1) == 1 && kv->size(0) % B == 0 && kv->size(1) >= 2 * Hkv * Dh,
                "attention: kv must be [B*Skv, 2*Hkv*Dh]");
    d.kv = kv->data_ptr();
    d.ld_kv = kv->stride(0);
    d.Skv = (int)(kv->size(0) / B);
    d.q_off = (int)q_off;
  }
  check(lk_attention_fwd(&d, stream()));
}

void attention_bwd(torch::Tensor qkv, torch::Tensor o, torch::Tensor dout, torch::Tensor lse,
                   torch::Tensor dqkv, torch::Tensor dq_acc, torch::Tensor dvec, int64_t B,
                   int64_t S, int64_t Hq, int64_t Hkv, int64_t Dh, bool causal, int64_t window,
                   double scale, torch::Tensor status) {
  const c10::cuda::CUDAGuard g(qkv.device());
  need(qkv, "qkv", torch::kBFloat16);
  need(o, "o", torch::kBFloat16);
  need(dout, "dout", torch::kBFloat16);
  need(dqkv, "dqkv", torch::kBFloat16);
  need_contig(lse, "lse", torch::kFloat32);
  need_contig(dq_acc, "dq_acc", torch::kFloat32);
  need_contig(dvec, "dvec", torch::kFloat32);
  TORCH_CHECK(dq_acc.numel() >= B * S * Hq * Dh && dvec.numel() >= 2 * ((B * Hq * S + 63) / 64 * 64), "attention_bwd: scratch too small");
  for (auto* t : {&qkv, &o, &dout, &dqkv})
    TORCH_CHECK(t->dim() == 2 && t->stride(1) == 1 && t->size(0) == B * S, "attention_bwd: bad 2-D operand");
  LkAttnBwdDesc d{};
  d.qkv = qkv.data_ptr(); d.ld_qkv = qkv.stride(0);
  d.o = o.data_ptr(); d.ld_o = o.stride(0);
  d.dout = dout.data_ptr(); d.ld_do = dout.stride(0);
  d.lse = lse.data_ptr<float>();
  d.dqkv = dqkv.data_ptr(); d.ld_dqkv = dqkv.stride(0);
  d.dq_acc = dq_acc.data_ptr<float>();
  d.dvec = dvec.data_ptr<float>();
  d.B = (int)B; d.S = (int)S; d.Hq = (int)Hq; d.Hkv = (int)Hkv; d.Dh = (int)Dh;
  d.causal = causal ? 1 : 0;
  d.window = (int)window;
  d.scale = (float)scale;
  d.status = status.data_ptr<int>();
  check(lk_attention_bwd(&d, stream()));
}

// ------------------------------------------------------ peer collectives
template <typename T>
T ptrs(const torch::Tensor& t) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == torch::kInt64, "pointer table must be a CUDA int64 tensor");
  return reinterpret_cast<T>(t.data_ptr());
}

void signal_barrier_dev(torch::Tensor sig_ptrs, int64_t rank, int64_t world, int64_t slot, torch::Tensor epoch_ctr,
                        torch::Tensor status) {
  const c10::cuda::CUDAGuard g(sig_ptrs.device());
  need(epoch_ctr, "epoch_ctr", torch::kInt32);
  check(lk_signal_barrier_dev(ptrs<int* const*>(sig_ptrs), (int)rank, (int)world, (int)slot,
                              epoch_ctr.data_ptr<int>(), status.data_ptr<int>(), stream()));
}

void signal_barrier(torch::Tensor sig_ptrs, int64_t rank, int64_t world, int64_t slot, int64_t epoch,
                    torch::Tensor status) {
  const c10::cuda::CUDAGuard g(sig_ptrs.device());
  check(lk_signal_barrier(ptrs<int* const*>(sig_ptrs), (int)rank, (int)world, (int)slot, (int)epoch,
                          status.data_ptr<int>(), stream()));
}

void allgather_copy(torch::Tensor src_ptrs, int64_t src_off_bytes, int64_t chunk_bytes, torch::Tensor dst,
                    int64_t world) {
  const c10::cuda::CUDAGuard g(dst.device());
  TORCH_CHECK(dst.is_contiguous() && dst.numel() * dst.element_size() >= chunk_bytes * world, "allgather: dst too small");
  check(lk_allgather_copy(ptrs<const void* const*>(src_ptrs), src_off_bytes, chunk_bytes, dst.data_ptr(),
                          (int)world, stream()));
}

void reduce_scatter_sum(torch::Tensor src_ptrs, int64_t src_off, int64_t n, torch::Tensor dst, int64_t world,
                        bool accumulate, c10::optional<torch::Tensor> partial) {
  const c10::cuda::CUDAGuard g(dst.device());
  need_contig(dst, "dst", torch::kFloat32);
  TORCH_CHECK(dst.numel() >= n, "reduce_scatter: dst too small");
  check(lk_reduce_scatter_sum(ptrs<const float* const*>(src_ptrs), src_off, n, dst.data_ptr<float>(),
                              (int)world, accumulate ? 1 : 0, optp<float>(partial),
                              partial.has_value() ? (int)partial->numel() : 0, stream()));
}

void reduce_scatter_bf16(torch::Tensor src_ptrs, int64_t src_off, int64_t n, torch::Tensor dst, int64_t world,
                         bool accumulate, c10::optional<torch::Tensor> partial) {
  const c10::cuda::CUDAGuard g(dst.device());
  need_contig(dst, "dst", torch::kFloat32);
  TORCH_CHECK(dst.numel() >= n, "reduce_scatter_bf16: dst too small");
  check(lk_reduce_scatter_bf16(ptrs<const void* const*>(src_ptrs), src_off, n, dst.data_ptr<float>(), (int)world,
                               accumulate ? 1 : 0, optp<float>(partial),
                               partial.has_value() ? (int)partial->numel() : 0, stream()));
}

void reduce_scatter_bf16_nvls(int64_t mc_ptr, int64_t n, torch::Tensor dst, bool accumulate,
                              c10::optional<torch::Tensor> partial) {
  const c10::cuda::CUDAGuard g(dst.device());
  need_contig(dst, "dst", torch::kFloat32);
  TORCH_CHECK(dst.numel() >= n, "reduce_scatter_bf16_nvls: dst too small");
  check(lk_reduce_scatter_bf16_nvls(reinterpret_cast<const void*>(mc_ptr), n, dst.data_ptr<float>(),
                                    accumulate ? 1 : 0, optp<float>(partial),
                                    partial.has_value() ? (int)partial->numel() : 0, stream()));
}

void allreduce_sum(torch::Tensor buf_ptrs, int64_t n, int64_t rank, int64_t world,
                   c10::optional<torch::Tensor> partial) {
  const c10::cuda::CUDAGuard g(buf_ptrs.device());
  check(lk_allreduce_sum(ptrs<float* const*>(buf_ptrs), n, (int)rank, (int)world, optp<float>(partial),
                         partial.has_value() ? (int)partial->numel() : 0, stream()));
}

void allreduce_sum_nvls(int64_t mc_ptr, int64_t n, int64_t rank, int64_t world,
                        c10::optional<torch::Tensor> partial, torch::Tensor like) {
  const c10::cuda::CUDAGuard g(like.device());
  check(lk_allreduce_sum_nvls(reinterpret_cast<float*>(mc_ptr), n, (int)rank, (int)world, optp<float>(partial),
                              partial.has_value() ? (int)partial->numel() : 0, stream()));
}

void reduce_scatter_sum_nvls(int64_t mc_ptr, int64_t n, torch::Tensor dst, bool accumulate,
                             c10::optional<torch::Tensor> partial) {
  const c10::cuda::CUDAGuard g(dst.device());
  need_contig(dst, "dst", torch::kFloat32);
  TORCH_CHECK(dst.numel() >= n, "reduce_scatter_nvls: dst too small");
  check(lk_reduce_scatter_sum_nvls(reinterpret_cast<const float*>(mc_ptr), n, dst.data_ptr<float>(),
                                   accumulate ? 1 : 0, optp<float>(partial),
                                   partial.has_value() ? (int)partial->numel() : 0, stream()));
}

void norm_exchange(torch::Tensor partial, torch::Tensor nbuf_ptrs, torch::Tensor sig_ptrs, int64_t rank,
                   int64_t world, int64_t slot, int64_t epoch, torch::Tensor state, double max_norm,
                   bool dynamic, double growth, double backoff, int64_t growth_interval, double min_scale,
                   torch::Tensor status) {
  const c10::cuda::CUDAGuard g(state.device());
  need_contig(partial, "partial", torch::kFloat32);
  need_contig(state, "state", torch::kFloat32);
  check(lk_norm_exchange(partial.data_ptr<float>(), (int)partial.numel(), ptrs<double* const*>(nbuf_ptrs),
                         ptrs<int* const*>(sig_ptrs), (int)rank, (int)world, (int)slot, (int)epoch,
                         state.data_ptr<float>(), (float)max_norm, dynamic ? 1 : 0, (float)growth,
                         (float)backoff, (int)growth_interval, (float)min_scale, status.data_ptr<int>(),
                         stream()));
}

// ---------------------------------------------------------------- serving
void kv_append(torch::Tensor qkv, int64_t Hq, int64_t Hkv, int64_t Dh, torch::Tensor slots,
               torch::Tensor k_cache, torch::Tensor v_cache, c10::optional<torch::Tensor> k_scale,
               c10::optional<torch::Tensor> v_scale, int64_t kv_dtype, torch::Tensor status) {
  const c10::cuda::CUDAGuard g(qkv.device());
  need(qkv, "qkv", torch::kBFloat16);
  TORCH_CHECK(qkv.dim() == 2 && qkv.stride(1) == 1, "kv_append: qkv must be row-major 2-D");
  need_contig(slots, "slots", torch::kInt32);
  TORCH_CHECK(k_cache.is_contiguous() && v_cache.is_contiguous(), "kv_append: caches must be contiguous");
  LkKvAppendDesc d{};
  d.qkv = qkv.data_ptr(); d.ld = qkv.stride(0); d.T = (int)qkv.size(0);
  d.Hq = (int)Hq; d.Hkv = (int)Hkv; d.Dh = (int)Dh;
  d.slots = slots.data_ptr<int>();
  d.k_cache = k_cache.data_ptr(); d.v_cache = v_cache.data_ptr();
  d.k_scale = optp<float>(k_scale); d.v_scale = optp<float>(v_scale);
  d.num_slots = (int)(k_cache.numel() / (Hkv * Dh));
  d.kv_dtype = (int)kv_dtype;
  d.status = status.data_ptr<int>();
  TORCH_CHECK(kv_dtype == 0 || (d.k_scale && d.v_scale), "kv_append: quantized caches need scales");
  check(lk_kv_append(&d, stream()));
}

void decode_attention(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache,
                      c10::optional<torch::Tensor> k_scale, c10::optional<torch::Tensor> v_scale,
                      torch::Tensor block_tables, torch::Tensor ctx_lens, int64_t block_size, int64_t Hq,
                      int64_t Hkv, int64_t Dh, double scale, int64_t split_len, int64_t num_splits,
                      c10::optional<torch::Tensor> part_o, c10::optional<torch::Tensor> part_ml,
                      torch::Tensor out, int64_t kv_dtype, c10::optional<torch::Tensor> status) {
  const c10::cuda::CUDAGuard g(q.device());
  need(q, "q", torch::kBFloat16);
  need(out, "out", torch::kBFloat16);
  need_contig(block_tables, "block_tables", torch::kInt32);
  need_contig(ctx_lens, "ctx_lens", torch::kInt32);
  LkDecodeDesc d{};
  d.q = q.data_ptr(); d.ldq = q.stride(0);
  d.k_cache = k_cache.data_ptr(); d.v_cache = v_cache.data_ptr();
  d.k_scale = optp<float>(k_scale); d.v_scale = optp<float>(v_scale);
  d.block_tables = block_tables.data_ptr<int>(); d.max_blocks = (int)block_tables.size(1);
  d.ctx_lens = ctx_lens.data_ptr<int>();
  d.block_size = (int)block_size; d.num_seqs = (int)q.size(0);
  d.Hq = (int)Hq; d.Hkv = (int)Hkv; d.Dh = (int)Dh; d.scale = (float)scale;
  d.split_len = (int)split_len; d.num_splits = (int)num_splits;
  d.part_o = optp<float>(part_o); d.part_ml = optp<float>(part_ml);
  d.out = out.data_ptr(); d.ldo = out.stride(0);
  d.kv_dtype = (int)kv_dtype;
  d.num_blocks = (int)(k_cache.numel() / (Hkv * Dh) / block_size);
  d.status = optp<int>(status);
  check(lk_decode_attention(&d, stream()));
}

void kv_gather(torch::Tensor k_cache, torch::Tensor v_cache, c10::optional<torch::Tensor> k_scale,
               c10::optional<torch::Tensor> v_scale, torch::Tensor slots, int64_t Hkv, int64_t Dh,
               torch::Tensor out, int64_t kv_dtype, c10::optional<torch::Tensor> status) {
  const c10::cuda::CUDAGuard g(out.device());
  need_contig(slots, "slots", torch::kInt32);
  need(out, "out", torch::kBFloat16);
  TORCH_CHECK(out.stride(1) == 1 && out.size(0) >= slots.numel(), "kv_gather: out shape");
  check(lk_kv_gather_checked(k_cache.data_ptr(), v_cache.data_ptr(), optp<float>(k_scale), optp<float>(v_scale),
                             slots.data_ptr<int>(), (int)slots.numel(), (int)Hkv, (int)Dh, out.data_ptr(),
                             out.stride(0), (int)kv_dtype, (int)(k_cache.numel() / (Hkv * Dh)),
                             optp<int>(status), stream()));
}

void sample(torch::Tensor logits, c10::optional<torch::Tensor> temperature, int64_t seed, torch::Tensor out_tok,
            c10::optional<torch::Tensor> out_val, int64_t v0) {
  const c10::cuda::CUDAGuard g(logits.device());
  need(logits, "logits", torch::kBFloat16);
  TORCH_CHECK(logits.dim() == 2 && logits.stride(1) == 1, "sample: logits must be row-major 2-D");
  need_contig(out_tok, "out_tok", torch::kInt64);
  check(lk_sample_vp(logits.data_ptr(), logits.stride(0), (int)logits.size(0), (int)logits.size(1), v0,
                     optp<float>(temperature), (uint64_t)seed, out_tok.data_ptr<int64_t>(), optp<float>(out_val),
                     stream()));
}

void sample_topp(torch::Tensor logits, torch::Tensor temperature, torch::Tensor top_p, int64_t seed,
                 c10::optional<torch::Tensor> row_seeds, torch::Tensor out_tok) {
  const c10::cuda::CUDAGuard g(logits.device());
  need(logits, "logits", torch::kBFloat16);
  TORCH_CHECK(logits.dim() == 2 && logits.stride(1) == 1, "sample_topp: logits must be row-major 2-D");
  need_contig(temperature, "temperature", torch::kFloat32);
  need_contig(top_p, "top_p", torch::kFloat32);
  need_contig(out_tok, "out_tok", torch::kInt64);
  const int64_t rows = logits.size(0);
  TORCH_CHECK(temperature.numel() >= rows && top_p.numel() >= rows && out_tok.numel() >= rows,
              "sample_topp: one temperature, top_p and output per row");
  const uint64_t* rs = nullptr;
  if (row_seeds.has_value()) {
    need_contig(*row_seeds, "row_seeds", torch::kInt64);
    TORCH_CHECK(row_seeds->numel() >= rows, "sample_topp: one seed per row");
    rs = reinterpret_cast<const uint64_t*>(row_seeds->data_ptr<int64_t>());
  }
  check(lk_sample_topp(logits.data_ptr(), logits.stride(0), (int)rows, (int)logits.size(1),
                       temperature.data_ptr<float>(), top_p.data_ptr<float>(), (uint64_t)seed, rs,
                       out_tok.data_ptr<int64_t>(), stream()));
}

void quantize(int64_t fmt, torch::Tensor w, int64_t group, torch::Tensor q, torch::Tensor scale,
              c10::optional<torch::Tensor> zero) {
  const c10::cuda::CUDAGuard g(w.device());
  need_contig(w, "w", torch::kBFloat16);
  need_contig(scale, "scale", torch::kFloat32);
  check(lk_quantize((int)fmt, w.data_ptr(), (int)w.size(0), (int)w.size(1), (int)group, q.data_ptr(),
                    scale.data_ptr<float>(), optp<float>(zero), stream()));
}

void dequant_gemv(int64_t fmt, torch::Tensor x, torch::Tensor q, torch::Tensor scale,
                  c10::optional<torch::Tensor> zero, int64_t N, int64_t K, int64_t group, torch::Tensor y) {
  const c10::cuda::CUDAGuard g(x.device());
  need(x, "x", torch::kBFloat16);
  need(y, "y", torch::kBFloat16);
  TORCH_CHECK(x.stride(1) == 1 && y.stride(1) == 1, "dequant_gemv: row-major x, y");
  check(lk_dequant_gemv((int)fmt, x.data_ptr(), x.stride(0), (int)x.size(0), q.data_ptr(), scale.data_ptr<float>(),
                        optp<float>(zero), (int)N, (int)K, (int)group, y.data_ptr(), y.stride(0), stream()));
}

void dequantize(int64_t fmt, torch::Tensor q, torch::Tensor scale, c10::optional<torch::Tensor> zero, int64_t N,
                int64_t K, int64_t group, torch::Tensor w) {
  const c10::cuda::CUDAGuard g(q.device());
  need_contig(w, "w", torch::kBFloat16);
  check(lk_dequantize((int)fmt, q.data_ptr(), scale.data_ptr<float>(), optp<float>(zero), (int)N, (int)K,
                      (int)group, w.data_ptr(), stream()));
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "lora_kernel_b200 sm_100a kernels";
  m.def("gemm", &gemm);
  m.def("gemm_rs", &gemm_rs);
  m.def("make_remote_maps", &make_remote_maps);
  m.def("gemm_ag", &gemm_ag);
  m.def("rs_sum", &rs_sum);
  m.def("gemm_gather", &gemm_gather);
  m.def("gemm_fp8", &gemm_fp8);
  m.def("quant_1x128", &quant_1x128);
  m.def("gemm_fp8_comm", &gemm_fp8_comm);
  m.def("dequant_1x128", &dequant_1x128);
  m.def("quant_128x128", &quant_128x128);
  m.def("gemm_mxf8", &gemm_mxf8);
  m.def("quant_mx_rows", &quant_mx_rows);
  m.def("quant_mx_128x128", &quant_mx_128x128);
  m.def("dequant_mx_rows", &dequant_mx_rows);
  m.def("dq_gemm", &dq_gemm);
  m.def("dq_gemm_splits", &dq_gemm_splits);
  m.def("allreduce_sum_nvls", &allreduce_sum_nvls);
  m.def("reduce_scatter_sum_nvls", &reduce_scatter_sum_nvls);
  m.def("cross_entropy_vp", &cross_entropy_vp);
  m.def("launch_count", []() { return (int64_t)lk_launch_count(); });
  m.def("rmsnorm_fwd", &rmsnorm_fwd);
  m.def("gelu_fwd", &gelu_fwd);
  m.def("dropout", &dropout);
  m.def("gelu_bwd", &gelu_bwd);
  m.def("layernorm_fwd", &layernorm_fwd);
  m.def("layernorm_bwd", &layernorm_bwd);
  m.def("rmsnorm_bwd", &rmsnorm_bwd);
  m.def("rmsnorm_bwd_partial_rows", &rmsnorm_bwd_partial_rows);
  m.def("rope", &rope);
  m.def("swiglu_fwd", &swiglu_fwd);
  m.def("swiglu_bwd", &swiglu_bwd);
  m.def("embedding_fwd", &embedding_fwd);
  m.def("embedding_bwd", &embedding_bwd);
  m.def("cross_entropy", &cross_entropy);
  m.def("adamw", &adamw);
  m.def("grad_norm_partials", &grad_norm_partials);
  m.def("optimizer_finalize", &optimizer_finalize);
  m.def("attention_fwd", &attention_fwd);
  m.def("signal_barrier", &signal_barrier);
  m.def("signal_barrier_dev", &signal_barrier_dev);
  m.def("kv_append", &kv_append);
  m.def("decode_attention", &decode_attention);
  m.def("sample", &sample);
  m.def("sample_topp", &sample_topp);
  m.def("kv_gather", &kv_gather);
  m.def("quantize", &quantize);
  m.def("dequant_gemv", &dequant_gemv);
  m.def("dequantize", &dequantize);
  m.def("allgather_copy", &allgather_copy);
  m.def("reduce_scatter_sum", &reduce_scatter_sum);
  m.def("cast_f32_bf16", &cast_f32_bf16);
  m.def("gemm_set_pair", [](int64_t mode) { lk_gemm_set_pair((int)mode); });
  m.def("gemm_pair_count", []() { return (int64_t)lk_gemm_pair_count(); });
  m.def("reduce_scatter_bf16", &reduce_scatter_bf16);
  m.def("reduce_scatter_bf16_nvls", &reduce_scatter_bf16_nvls);
  m.def("allreduce_sum", &allreduce_sum);
  m.def("norm_exchange", &norm_exchange);
  m.attr("SIG_SLOTS") = (int)LK_SIG_SLOTS;
  m.def("attention_bwd", &attention_bwd);
  m.attr("EPI_BF16") = (int)LK_EPI_BF16;
  m.attr("EPI_F32") = (int)LK_EPI_F32;
  m.attr("EPI_F32_ACC") = (int)LK_EPI_F32_ACC;
  m.attr("EPI_BF16_RESID") = (int)LK_EPI_BF16_RESID;
  m.attr("EPI_SWIGLU") = (int)LK_EPI_SWIGLU;
}
