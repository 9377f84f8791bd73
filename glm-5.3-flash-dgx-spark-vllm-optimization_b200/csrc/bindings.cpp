#include <cstdlib>
// Python bindings of the glm53 CUDA kernels (torch tensors -> raw pointers; launches on the current stream).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "launchers.h"

#include <mutex>
#include <vector>

// Bounds-checked debug build: every CUDA source registers its device error record here at load time (see
// common.cuh); bounds_status() reads them, bounds_reset() clears them.  The regular build registers none.
struct G53BoundsRecHost {
  int count;
  int code;
  long long index;
  long long limit;
};
static std::vector<const void*>& g53_bounds_symbols() {
  static std::vector<const void*> v;
  return v;
}
static std::mutex g53_bounds_mu;
void g53_bounds_register(const void* symbol) {
  std::lock_guard<std::mutex> lock(g53_bounds_mu);
  g53_bounds_symbols().push_back(symbol);
}

namespace {

using at::Tensor;
using OptT = c10::optional<Tensor>;

void check(cudaError_t e, const char* what) {
  TORCH_CHECK(e == cudaSuccess, "glm53 kernel ", what, " failed: ", cudaGetErrorString(e));
}

template <class T>
T* P(const Tensor& t) { return reinterpret_cast<T*>(t.data_ptr()); }
template <class T>
T* P(const OptT& t) { return (t.has_value() && t->defined()) ? reinterpret_cast<T*>(t->data_ptr()) : nullptr; }

cudaStream_t stream() { return at::cuda::getCurrentCUDAStream().stream(); }

void cuda_check(const Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
}

// ------------------------------------------------------------------------------------------------- GEMV
Tensor& err_word(const Tensor& like);

void gemv(const Tensor& x, const Tensor& w, const OptT& scale, const Tensor& y, int64_t mode, double limit,
          int64_t ks, int64_t cl) {
  cuda_check(x, "x"); cuda_check(w, "w"); cuda_check(y, "y");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16, "x must be bf16");
  TORCH_CHECK(x.stride(-1) == 1 && w.stride(-1) == 1 && y.stride(-1) == 1, "inner dims must be contiguous");
  const bool batched = w.dim() == 3;
  TORCH_CHECK(x.dim() == (batched ? 3 : 2) && y.dim() == x.dim(), "rank mismatch");
  GemvArgs p{};
  p.x = P<const __nv_bfloat16>(x);
  p.w = w.data_ptr();
  p.scale = P<const float>(scale);
  p.y = y.data_ptr();
  p.batch = batched ? (int)w.size(0) : 1;
  p.M = (int)x.size(-2);
  p.K = (int)x.size(-1);
  p.N = (int)w.size(-2);
  TORCH_CHECK(w.size(-1) == p.K, "K mismatch: x ", p.K, " w ", w.size(-1));
  p.ldx = x.stride(-2);
  p.bsx = batched ? x.stride(0) : 0;
  // 16-byte vector loads of activations and weights: refuse operands that would fault
  TORCH_CHECK(reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0 && p.ldx % 8 == 0 && p.bsx % 8 == 0,
              "gemv: activation rows must start on 16-byte boundaries (row stride ", p.ldx, ")");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(w.data_ptr()) % 16 == 0, "gemv: weights must be 16-byte aligned");
  p.push_ptrs = nullptr;
  p.bsw = batched ? w.stride(0) : 0;
  p.bss = (batched && scale.has_value()) ? scale->stride(0) : 0;
  p.ldy = y.stride(-2);
  p.bsy = batched ? y.stride(0) : 0;
  p.mode = (int)mode;
  p.limit = (float)limit;
  if (mode == GEMV_BF16 || mode == GEMV_SWIGLU) {
    TORCH_CHECK(y.scalar_type() == at::kBFloat16, "y must be bf16");
  } else {
    TORCH_CHECK(y.scalar_type() == at::kFloat, "y must be fp32");
  }
  TORCH_CHECK(y.size(-2) >= p.M, "y rows");
  if (w.scalar_type() == at::kByte || w.scalar_type() == at::kFloat8_e4m3fn) {
    TORCH_CHECK(scale.has_value(), "fp8 weights need a scale");
    p.force_ks = (int)ks;
    p.force_cl = (int)cl;
    p.err = err_word(x).data_ptr<int>();
    check(g53_gemv_fp8(p, stream()), "gemv_fp8");
  } else {
    TORCH_CHECK(w.scalar_type() == at::kBFloat16, "weights must be fp8 (uint8) or bf16");
    check(g53_gemv_bf16(p, stream()), "gemv_bf16");
  }
}

// ------------------------------------------------------------------------------------------------- GEMM
Tensor& err_word(const Tensor& like) {
  static std::vector<Tensor> words(64);
  const int dev = like.get_device();
  if (!words[dev].defined()) words[dev] = torch::zeros({4}, like.options().dtype(at::kInt));
  return words[dev];
}

// a [M, K] or [B, M, K], w [N, K] or [B, N, K], y [M, N] or [B, M, N]; rows K-major (inner stride 1), batch and
// row strides free (e.g. per-head views of [rows, heads, dim] activations)
void gemm_common(const Tensor& a, bool fp8, const OptT& a_scale, const Tensor& w, const OptT& w_scale, const Tensor& y,
                 int64_t mode, double limit) {
  const bool bat = a.dim() == 3;
  TORCH_CHECK(w.dim() == a.dim() && y.dim() == a.dim(), "a, w and y must all be 2-D or all 3-D");
  TORCH_CHECK(a.stride(-1) == 1 && w.stride(-1) == 1 && y.stride(-1) == 1, "rows must be contiguous");
  GemmArgs p{};
  p.a = a.data_ptr(); p.lda = a.stride(-2);
  p.b = w.data_ptr(); p.ldb = w.stride(-2);
  p.a_scale = P<const float>(a_scale);
  p.b_scale = P<const float>(w_scale);
  p.y = y.data_ptr(); p.ldy = y.stride(-2);
  p.M = (int)a.size(-2); p.N = (int)w.size(-2); p.K = (int)a.size(-1);
  p.mode = (int)mode; p.fp8 = fp8 ? 1 : 0; p.limit = (float)limit;
  p.err = P<int>(err_word(a));
  if (bat) {
    TORCH_CHECK(w.size(0) == a.size(0) && y.size(0) == a.size(0), "batch mismatch");
    p.batch = (int)a.size(0);
    p.bsa = a.stride(0); p.bsb = w.stride(0); p.bsy = y.stride(0);
    if (w_scale.has_value()) {
      TORCH_CHECK(w_scale->dim() == 2 && w_scale->stride(1) == 1, "batched scales must be [B, N]");
      p.bss = w_scale->stride(0);
    }
  }
  TORCH_CHECK(w.size(-1) == p.K, "K mismatch");
  TORCH_CHECK(y.size(-2) == p.M, "y rows mismatch");
  if (mode == GEMV_BF16 || mode == GEMV_SWIGLU) {
    TORCH_CHECK(y.scalar_type() == at::kBFloat16, "y must be bf16");
  } else {
    TORCH_CHECK(y.scalar_type() == at::kFloat, "y must be fp32");
  }
  check(g53_gemm_sm100(p, stream()), "gemm_sm100");
}

// W8A8: bf16 activations quantised per row to e4m3, fp8 weights with per-row scales
void gemm_w8(const Tensor& x, const Tensor& w, const Tensor& scale, const Tensor& y, int64_t mode, double limit) {
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.stride(1) == 1);
  const int64_t M = x.size(0), K = x.size(1);
  auto q = torch::empty({M, K}, x.options().dtype(at::kByte));
  auto qs = torch::empty({M}, x.options().dtype(at::kFloat));
  check(g53_quant_rows_e4m3(P<const __nv_bfloat16>(x), x.stride(0), (int)M, (int)K, P<uint8_t>(q), P<float>(qs),
                            stream()),
        "quant_rows_e4m3");
  gemm_common(q, true, qs, w, scale, y, mode, limit);
}

// per-row e4m3 quantisation of bf16 rows (the W8A8 activation format: q [M, K] uint8, qs [M] fp32).  A row's
// codes depend on that row only, so rows quantised on their own rank and all-gathered equal rows gathered first
void quant_rows(const Tensor& x, const Tensor& q, const Tensor& qs) {
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.stride(1) == 1);
  TORCH_CHECK(q.scalar_type() == at::kByte && q.is_contiguous() && q.size(0) == x.size(0) && q.size(1) == x.size(1),
              "q must be uint8 [M, K], contiguous");
  TORCH_CHECK(qs.scalar_type() == at::kFloat && qs.numel() >= x.size(0), "qs must be fp32 [M]");
  check(g53_quant_rows_e4m3(P<const __nv_bfloat16>(x), x.stride(0), (int)x.size(0), (int)x.size(1), P<uint8_t>(q),
                            P<float>(qs), stream()),
        "quant_rows_e4m3");
}

// W8A8 GEMM of rows already in the e4m3 row format (quant_rows): the sequence-parallel prefill all-gathers the
// quantised rows of the KDA input projection instead of bf16 rows
void gemm_w8q(const Tensor& q, const Tensor& qs, const Tensor& w, const Tensor& scale, const Tensor& y, int64_t mode,
              double limit) {
  TORCH_CHECK(q.scalar_type() == at::kByte && q.dim() == 2 && q.stride(1) == 1);
  TORCH_CHECK(qs.scalar_type() == at::kFloat && qs.numel() >= q.size(0));
  gemm_common(q, true, qs, w, scale, y, mode, limit);
}

// W8A16: the fp8 weight widened exactly to bf16 in a scratch, then the bf16 tcgen05 GEMM with the per-row
// weight scales applied in the epilogue (same numerics as the small-M kernel: bf16 activations, exact weights)
void gemm_w8a16(const Tensor& x, const Tensor& w, const Tensor& scale, const Tensor& y, int64_t mode, double limit,
                const Tensor& scratch) {
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.stride(-1) == 1);
  TORCH_CHECK(scratch.scalar_type() == at::kBFloat16 && scratch.numel() >= w.numel(), "scratch too small");
  TORCH_CHECK(w.is_contiguous());
  check(g53_e4m3_to_bf16(P<const uint8_t>(w), w.numel(), P<__nv_bfloat16>(scratch), stream()), "e4m3_to_bf16");
  auto wb = scratch.flatten().narrow(0, 0, w.numel()).view(w.sizes());
  gemm_common(x, false, {}, wb, scale, y, mode, limit);
}

void gemm_bf16(const Tensor& x, const Tensor& w, const OptT& scale, const Tensor& y, int64_t mode, double limit) {
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16);
  gemm_common(x, false, {}, w, scale, y, mode, limit);
}

// W8A16 GEMM whose fp32 output rows are also stored into every rank's receive slot (fused tensor-parallel
// reduction at prefill; the consumer is hc_post_pre_tp)
void gemm_w8a16_push(const Tensor& x, const Tensor& w, const Tensor& scale, const Tensor& y, int64_t mode,
                     const Tensor& scratch, const Tensor& push_ptrs, const Tensor& push_flags, const Tensor& push_done,
                     int64_t slot, int64_t rank, int64_t world) {
  TORCH_CHECK(mode == GEMV_F32 || mode == GEMV_F32_ACC, "push needs an fp32 output mode");
  TORCH_CHECK(x.dim() == 2 && y.is_contiguous() && y.stride(0) * y.size(0) <= slot);
  TORCH_CHECK(scratch.scalar_type() == at::kBFloat16 && scratch.numel() >= w.numel(), "scratch too small");
  check(g53_e4m3_to_bf16(P<const uint8_t>(w), w.numel(), P<__nv_bfloat16>(scratch), stream()), "e4m3_to_bf16");
  auto wb = scratch.flatten().narrow(0, 0, w.numel()).view(w.sizes());
  GemmArgs p{};
  p.a = x.data_ptr(); p.lda = x.stride(0);
  p.b = wb.data_ptr(); p.ldb = wb.stride(0);
  p.b_scale = P<const float>(scale);
  p.y = y.data_ptr(); p.ldy = y.stride(0);
  p.M = (int)x.size(0); p.N = (int)w.size(0); p.K = (int)x.size(1);
  p.mode = (int)mode; p.fp8 = 0;
  p.err = P<int>(err_word(x));
  p.push_ptrs = reinterpret_cast<float* const*>(push_ptrs.data_ptr());
  p.push_flags = reinterpret_cast<unsigned* const*>(push_flags.data_ptr());
  p.push_done = reinterpret_cast<unsigned*>(push_done.data_ptr());
  p.push_slot = slot; p.push_rank = (int)rank; p.push_world = (int)world;
  check(g53_gemm_sm100(p, stream()), "gemm_w8a16_push");
}

// all-gather + GEMM (column-parallel input): y [W * rows, N] = A_all @ (w8 * s)^T with A row-sharded over the ranks;
// shard j at ptrs[j] (host int64 list of device addresses, peer memory), row pitch lda; waits (bounded) for
// flags[j] >= target (raised by rank j's signal_peers after it wrote its shard)
void gemm_ag_w8a16(const Tensor& ptrs, const Tensor& ptrs_dev, int64_t rank, int64_t rows, int64_t K, int64_t lda,
                   const Tensor& w, const Tensor& scale, const Tensor& y, int64_t mode, const Tensor& scratch,
                   const Tensor& flags, int64_t target, const Tensor& stage, const Tensor& ready) {
  TORCH_CHECK(ptrs.device().is_cpu() && ptrs.scalar_type() == at::kLong, "ptrs: host int64 addresses");
  TORCH_CHECK(scratch.scalar_type() == at::kBFloat16 && scratch.numel() >= w.numel(), "scratch too small");
  TORCH_CHECK(flags.scalar_type() == at::kInt && flags.numel() >= ptrs.numel());
  const int W = (int)ptrs.numel();
  check(g53_e4m3_to_bf16(P<const uint8_t>(w), w.numel(), P<__nv_bfloat16>(scratch), stream()), "e4m3_to_bf16");
  auto wb = scratch.flatten().narrow(0, 0, w.numel()).view(w.sizes());
  GemmArgs p{};
  p.a = nullptr; p.lda = lda;
  p.b = wb.data_ptr(); p.ldb = wb.stride(0);
  p.b_scale = P<const float>(scale);
  p.y = y.data_ptr(); p.ldy = y.stride(0);
  p.M = (int)(W * rows); p.N = (int)w.size(0); p.K = (int)K;
  p.mode = (int)mode; p.fp8 = 0;
  p.err = P<int>(err_word(y));
  p.ag_world = W; p.ag_rows = (int)rows; p.ag_rank = (int)rank; p.ag_ptrs = ptrs.data_ptr<int64_t>();
  p.ag_ptrs_dev = P<const int64_t>(ptrs_dev);
  p.ag_flags = reinterpret_cast<const unsigned*>(flags.data_ptr()); p.ag_target = (unsigned)target;
  TORCH_CHECK(stage.scalar_type() == at::kBFloat16 && stage.numel() >= (int64_t)W * rows * K, "stage too small");
  TORCH_CHECK(ready.scalar_type() == at::kInt && ready.numel() >= (int64_t)W * rows / 128, "ready too small");
  p.ag_stage = P<__nv_bfloat16>(stage);
  p.ag_ready = P<int>(ready);
  TORCH_CHECK(y.size(0) == p.M && y.size(1) == p.N && y.stride(1) == 1, "y must be [W * rows, N]");
  check(g53_gemm_sm100(p, stream()), "gemm_ag_w8a16");
}

void signal_peers(const Tensor& flag_addrs, int64_t rank) {
  TORCH_CHECK(flag_addrs.scalar_type() == at::kLong && flag_addrs.is_cuda());
  check(g53_signal_peers(P<const int64_t>(flag_addrs), (int)rank, (int)flag_addrs.numel(), stream()), "signal_peers");
}

int64_t gemm_error(const Tensor& like) {
  auto& e = err_word(like);
  const int64_t v = e[0].item<int>();
  e.zero_();
  return v;
}

// fused tensor-parallel variant: the fp32 partial is also pushed into every rank's receive slot (peer memory)
void gemv_push(const Tensor& x, const Tensor& w, const Tensor& scale, const Tensor& y, int64_t mode,
               const Tensor& push_ptrs, const Tensor& push_flags, const Tensor& push_done, int64_t slot, int64_t rank,
               int64_t world, const Tensor& err) {
  TORCH_CHECK(mode == GEMV_F32 || mode == GEMV_F32_ACC, "push needs an fp32 output mode");
  TORCH_CHECK(w.dim() == 2 && x.dim() == 2 && y.is_contiguous() && y.stride(0) * y.size(0) <= slot);
  GemvArgs p{};
  p.x = P<const __nv_bfloat16>(x);
  p.w = w.data_ptr();
  p.scale = P<const float>(scale);
  p.y = y.data_ptr();
  p.batch = 1;
  p.M = (int)x.size(0);
  p.K = (int)x.size(1);
  p.N = (int)w.size(0);
  p.ldx = x.stride(0);
  p.ldy = y.stride(0);
  p.mode = (int)mode;
  TORCH_CHECK(reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0 && p.ldx % 8 == 0, "gemv: misaligned activations");
  p.push_ptrs = reinterpret_cast<float* const*>(push_ptrs.data_ptr());
  p.push_flags = reinterpret_cast<unsigned* const*>(push_flags.data_ptr());
  p.push_done = reinterpret_cast<unsigned*>(push_done.data_ptr());
  p.push_slot = slot;
  p.push_rank = (int)rank;
  p.push_world = (int)world;
  p.err = P<int>(err);
  check(g53_gemv_fp8(p, stream()), "gemv_push");
}

// the byte ranges of the given tensors, in order, at most max_bytes in total (at most four tensors)
L2Ranges l2_ranges(const std::vector<Tensor>& ts, int64_t max_bytes) {
  L2Ranges r{};
  int64_t left = max_bytes;
  for (const auto& t : ts) {
    if (r.count == 4 || left <= 0) break;
    cuda_check(t, "prefetched tensor");
    TORCH_CHECK(t.is_contiguous(), "l2_prefetch: tensors must be contiguous");
    const int64_t n = std::min<int64_t>(left, t.numel() * t.element_size());
    r.ptr[r.count] = reinterpret_cast<const char*>(t.data_ptr());
    r.bytes[r.count] = n;
    ++r.count;
    left -= n;
  }
  return r;
}

// prefetch the given tensors into L2 from a separate small kernel
void l2_prefetch(const std::vector<Tensor>& ts, int64_t max_bytes) {
  check(g53_l2_prefetch(l2_ranges(ts, max_bytes), stream()), "l2_prefetch");
}

// grouped dynamic conv of the block drafter: x [T, H] bf16, delta [T, taps, H/gs] bf16, base [taps, H] bf16
void dconv(const Tensor& x, const Tensor& delta, const Tensor& base, const Tensor& out, int64_t gs,
           int64_t block_size) {
  cuda_check(x, "x"); cuda_check(delta, "delta"); cuda_check(base, "base"); cuda_check(out, "out");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && delta.scalar_type() == at::kBFloat16 &&
              base.scalar_type() == at::kBFloat16 && out.scalar_type() == at::kBFloat16, "dconv: bf16 tensors");
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1 && x.stride(0) % 2 == 0, "dconv: x [T, H], unit inner stride");
  const int64_t T = x.size(0), H = x.size(1);
  TORCH_CHECK(base.dim() == 2 && base.size(1) == H && base.is_contiguous(), "dconv: base [taps, H] contiguous");
  const int64_t taps = base.size(0);
  TORCH_CHECK(gs >= 1 && H % gs == 0 && H % 2 == 0, "dconv: H must be even and a multiple of gs");
  TORCH_CHECK(delta.is_contiguous() && delta.numel() == T * taps * (H / gs), "dconv: delta [T, taps, H/gs]");
  TORCH_CHECK(out.is_contiguous() && out.size(0) == T && out.size(1) == H, "dconv: out [T, H] contiguous");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(x.data_ptr()) % 4 == 0 && reinterpret_cast<uintptr_t>(base.data_ptr()) % 4 == 0 &&
              reinterpret_cast<uintptr_t>(out.data_ptr()) % 4 == 0, "dconv: 4-byte aligned rows");
  DconvArgs a{};
  a.x = P<const __nv_bfloat16>(x); a.ldx = x.stride(0);
  a.delta = P<const __nv_bfloat16>(delta);
  a.base = P<const __nv_bfloat16>(base);
  a.out = P<__nv_bfloat16>(out);
  a.T = (int)T; a.H = (int)H; a.taps = (int)taps; a.gs = (int)gs; a.G = (int)(H / gs);
  a.block_size = (int)block_size;
  check(g53_dconv(a, stream()), "dconv");
}

// ------------------------------------------------------------------------------------------------- MoE
void moe_route(const Tensor& logits, const Tensor& bias, int64_t top_k, double scale, bool norm,
               const Tensor& topk_ids, const Tensor& topk_w, const Tensor& group_count, const Tensor& group_expert,
               const Tensor& group_offset, const Tensor& pair_token, const Tensor& pair_expert, const Tensor& pair_w,
               const Tensor& pair_of) {
  RouteArgs a{};
  a.logits = P<const float>(logits);
  a.bias = P<const float>(bias);
  a.R = (int)logits.size(0);
  a.E = (int)logits.size(1);
  a.top_k = (int)top_k;
  a.scale = (float)scale;
  a.norm = norm ? 1 : 0;
  a.topk_ids = P<int>(topk_ids);
  a.topk_w = P<float>(topk_w);
  a.group_count = P<int>(group_count);
  a.group_expert = P<int>(group_expert);
  a.group_offset = P<int>(group_offset);
  a.pair_token = P<int>(pair_token);
  a.pair_expert = P<int>(pair_expert);
  a.pair_w = P<float>(pair_w);
  a.pair_of = P<int>(pair_of);
  a.max_groups = (int)group_expert.size(0);
  TORCH_CHECK(group_offset.size(0) >= a.max_groups + 1, "group_offset too small");
  check(g53_moe_route(a, stream()), "moe_route");
}

Exl3Args exl3_args(const Tensor& x, const Tensor& tr_g, const Tensor& suh_g, const Tensor& svh_g, const Tensor& tr_u,
                   const Tensor& suh_u, const Tensor& svh_u, const Tensor& tr_d, const Tensor& suh_d,
                   const Tensor& svh_d, const Tensor& group_count, const Tensor& group_expert,
                   const Tensor& group_offset, const Tensor& pair_token, const Tensor& pair_expert,
                   const Tensor& pair_w, const Tensor& xh_g, const Tensor& xh_u, const Tensor& xd, const Tensor& yd,
                   double limit) {
  Exl3Args a{};
  a.x = P<const __nv_bfloat16>(x);
  a.ldx = x.stride(0);
  a.tr_g = P<const int16_t>(tr_g); a.suh_g = P<const __half>(suh_g); a.svh_g = P<const __half>(svh_g);
  a.tr_u = P<const int16_t>(tr_u); a.suh_u = P<const __half>(suh_u); a.svh_u = P<const __half>(svh_u);
  a.tr_d = P<const int16_t>(tr_d); a.suh_d = P<const __half>(suh_d); a.svh_d = P<const __half>(svh_d);
  a.K = (int)suh_g.size(-1);
  a.N = (int)svh_g.size(-1);
  a.Dout = (int)svh_d.size(-1);
  a.group_count = P<const int>(group_count);
  a.group_expert = P<const int>(group_expert);
  a.group_offset = P<const int>(group_offset);
  a.pair_token = P<const int>(pair_token);
  a.pair_expert = P<const int>(pair_expert);
  a.pair_w = P<const float>(pair_w);
  a.max_groups = (int)group_expert.size(0);
  a.pairs = (int)pair_token.size(0);
  a.limit = (float)limit;
  a.xh_g = P<__half>(xh_g); a.xh_u = P<__half>(xh_u); a.xd = P<__half>(xd); a.yd = P<float>(yd);
  a.decode_layout = 1;
  a.n_rows = x.size(0);
  a.n_experts = tr_g.size(0);
  TORCH_CHECK(tr_g.scalar_type() == at::kShort && tr_d.scalar_type() == at::kShort, "trellis must be int16");
  // decode layout: rotated inputs are duplicated f16 pairs, 2K (2N) halves per pair
  TORCH_CHECK(xh_g.numel() >= (int64_t)a.pairs * 2 * a.K && xh_u.numel() >= (int64_t)a.pairs * 2 * a.K &&
                  xd.numel() >= (int64_t)a.pairs * 2 * a.N && yd.size(0) >= a.pairs,
              "exl3_moe scratch too small (xh: pairs x 2K halves, xd: pairs x 2N halves)");
  return a;
}

void exl3_moe(const Tensor& x, const Tensor& tr_g, const Tensor& suh_g, const Tensor& svh_g, const Tensor& tr_u,
              const Tensor& suh_u, const Tensor& svh_u, const Tensor& tr_d, const Tensor& suh_d, const Tensor& svh_d,
              const Tensor& group_count, const Tensor& group_expert, const Tensor& group_offset,
              const Tensor& pair_token, const Tensor& pair_expert, const Tensor& pair_w, const Tensor& xh_g,
              const Tensor& xh_u, const Tensor& xd, const Tensor& yd, double limit,
              const std::vector<Tensor>& prefetch, int64_t prefetch_bytes) {
  Exl3Args a = exl3_args(x, tr_g, suh_g, svh_g, tr_u, suh_u, svh_u, tr_d, suh_d, svh_d, group_count, group_expert,
                         group_offset, pair_token, pair_expert, pair_w, xh_g, xh_u, xd, yd, limit);
  a.pf = l2_ranges(prefetch, prefetch_bytes);
  check(g53_exl3_rot_in(a, stream()), "exl3_rot_in");
  check(g53_exl3_gate_up(a, stream()), "exl3_gate_up");
  check(g53_exl3_down(a, stream()), "exl3_down");
}

// Expert-parallel MoE step (ep_moe.cu): dispatch -> plan -> rot_in -> gate_up -> down (epilogue stores into the
// sources' combine rows) -> combine.  `peer` int64 [6, world] (device): addresses on every rank of recv_x, recv_meta,
// recv_cnt, disp_flag[p][rank], comb, comb_flag[p][rank]; `local` int64 [6] (host): this rank's disp_flag[p],
// comb_flag[p], recv_cnt, recv_meta, comb, recv_x of parity p; `state` int32 [16] (device, parity p): counters
// (0 dispatch, 1 down, 2 combine), 3 pair count, 4 received rows, 5 epoch, 8 error code.
void ep_moe_step(const Tensor& x, const Tensor& out, const Tensor& pair_token, const Tensor& pair_expert,
                 const Tensor& pair_w, const Tensor& pair_of, const Tensor& tr_g, const Tensor& suh_g,
                 const Tensor& svh_g, const Tensor& tr_u, const Tensor& suh_u, const Tensor& svh_u, const Tensor& tr_d,
                 const Tensor& suh_d, const Tensor& svh_d, const Tensor& peer, const Tensor& local, const Tensor& state,
                 const Tensor& seg, const Tensor& groups, const Tensor& rp_i, const Tensor& rp_w, const Tensor& rp_out,
                 const Tensor& xh_g, const Tensor& xh_u, const Tensor& xd, int64_t El, int64_t rank, int64_t world,
                 int64_t cap, int64_t recv_cap, int64_t top_k, double limit, bool tensor_core_experts) {
  const int T = (int)x.size(0), K = (int)x.size(1), W = (int)world;
  TORCH_CHECK(peer.dim() == 2 && peer.size(0) == 6 && peer.size(1) == W && peer.scalar_type() == at::kLong);
  TORCH_CHECK(local.device().is_cpu() && local.numel() == 6 && local.scalar_type() == at::kLong);
  TORCH_CHECK(state.numel() >= 16 && state.scalar_type() == at::kInt);
  TORCH_CHECK(T * top_k <= cap && W * El <= 1024 && out.scalar_type() == at::kFloat);
  TORCH_CHECK(xh_g.numel() >= recv_cap * 2 * K && xd.numel() >= recv_cap * 2 * svh_g.size(-1), "EP scratch");
  const int64_t* pp = P<const int64_t>(peer);
  const int64_t* lp = local.data_ptr<int64_t>();
  int* st = P<int>(state);
  EpArgs e{};
  e.n_pairs = st + 3;
  e.pair_token = P<const int>(pair_token); e.pair_expert = P<const int>(pair_expert); e.pair_w = P<const float>(pair_w);
  e.x = P<const __nv_bfloat16>(x); e.ldx = x.stride(0);
  e.K = K; e.El = (int)El; e.rank = (int)rank; e.world = W; e.cap = (int)cap; e.recv_cap = (int)recv_cap;
  e.recv_x = pp; e.recv_meta = pp + W; e.recv_cnt = pp + 2 * W; e.disp_flags = pp + 3 * W; e.comb = pp + 4 * W;
  e.done = reinterpret_cast<unsigned*>(st + 0); e.done2 = reinterpret_cast<unsigned*>(st + 2);
  e.epoch = reinterpret_cast<unsigned*>(st + 5);
  e.err = st + 8;
  e.my_disp_flags = reinterpret_cast<const unsigned*>(lp[0]);
  e.my_comb_flags = reinterpret_cast<const unsigned*>(lp[1]);
  e.my_cnt = reinterpret_cast<const int*>(lp[2]);
  e.my_meta = reinterpret_cast<const void*>(lp[3]);
  e.my_comb = reinterpret_cast<const float*>(lp[4]);
  int* sg = P<int>(seg);
  e.seg_base = sg; e.seg_cnt = sg + W * El; e.seg_src = sg + 2 * W * El;
  e.n_recv = st + 4;
  int* gr = P<int>(groups);
  e.group_count = gr; e.group_expert = gr + 1; e.group_offset = gr + 1 + El;
  e.rp_token = P<int>(rp_i); e.rp_expert = P<int>(rp_i) + recv_cap; e.rp_w = P<float>(rp_w);
  e.rp_out = P<int64_t>(rp_out);
  cudaStream_t s = stream();
  // state[3] holds this step's pair count (T * top_k), set by the caller
  check(g53_ep_dispatch(e, (int)(T * top_k), s), "ep_dispatch");
  check(g53_ep_plan(e, s), "ep_plan");
  Exl3Args a{};
  a.x = reinterpret_cast<const __nv_bfloat16*>(lp[5]); a.ldx = K;
  a.tr_g = P<const int16_t>(tr_g); a.suh_g = P<const __half>(suh_g); a.svh_g = P<const __half>(svh_g);
  a.tr_u = P<const int16_t>(tr_u); a.suh_u = P<const __half>(suh_u); a.svh_u = P<const __half>(svh_u);
  a.tr_d = P<const int16_t>(tr_d); a.suh_d = P<const __half>(suh_d); a.svh_d = P<const __half>(svh_d);
  a.K = K; a.N = (int)svh_g.size(-1); a.Dout = (int)svh_d.size(-1);
  a.n_experts = tr_g.size(0);
  a.group_count = e.group_count; a.group_expert = e.group_expert; a.group_offset = e.group_offset;
  a.pair_token = e.rp_token; a.pair_expert = e.rp_expert; a.pair_w = e.rp_w;
  a.max_groups = (int)El; a.pairs = (int)recv_cap; a.limit = (float)limit;
  a.xh_g = P<__half>(xh_g); a.xh_u = P<__half>(xh_u); a.xd = P<__half>(xd); a.yd = nullptr;
  a.decode_layout = tensor_core_experts ? 0 : 1;
  a.pair_count = e.n_recv;
  // the receiver's group count is only known on the device: bounded grid rows, CTAs stride over the groups
  a.launch_groups = (int)std::min<int64_t>(El, std::max<int64_t>(8, (int64_t)W * T * top_k));
  check(g53_exl3_rot_in(a, s), "ep rot_in");
  if (!tensor_core_experts) {
    // few rows per expert: trellis decoded in registers (mma.sync)
    check(g53_exl3_gate_up(a, s), "ep gate_up");
    a.out_ptrs = e.rp_out;
    a.done = reinterpret_cast<unsigned*>(st + 1);
    a.push_flags = pp + 5 * W;
    a.push_world = W;
    check(g53_exl3_down(a, s), "ep down");
  } else {
    // many rows per expert: tcgen05 grouped GEMMs with the trellis decoded into shared memory
    MoePrefillArgs q{};
    q.tr0 = a.tr_g; q.tr1 = a.tr_u; q.svh0 = a.svh_g; q.svh1 = a.svh_u; q.suh_next = a.suh_d;
    q.group_count = e.group_count; q.group_expert = e.group_expert; q.group_offset = e.group_offset;
    q.x0 = a.xh_g; q.x1 = a.xh_u; q.rows = recv_cap; q.K = K; q.N = a.N; q.max_groups = (int)El;
    q.out = a.xd; q.limit = (float)limit; q.err = st + 8;
    check(g53_moe_prefill(q, true, s), "ep moe_prefill gate_up");
    MoePrefillArgs r{};
    r.tr0 = a.tr_d; r.tr1 = a.tr_d; r.svh0 = a.svh_d; r.pair_w = e.rp_w;
    r.group_count = e.group_count; r.group_expert = e.group_expert; r.group_offset = e.group_offset;
    r.x0 = a.xd; r.rows = recv_cap; r.K = a.N; r.N = a.Dout; r.max_groups = (int)El;
    r.out = nullptr; r.limit = (float)limit; r.err = st + 8;
    r.out_ptrs = e.rp_out;
    r.done = reinterpret_cast<unsigned*>(st + 1);
    r.push_flags = pp + 5 * W;
    r.push_world = W;
    check(g53_moe_prefill(r, false, s), "ep moe_prefill down");
  }
  check(g53_ep_combine(e, P<const int>(pair_of), T, (int)top_k, P<float>(out), s), "ep_combine");
}

void exl3_rot_in(const Tensor& x, const Tensor& suh_g, const Tensor& suh_u, const Tensor& pair_token,
                 const Tensor& pair_expert, const Tensor& xh_g, const Tensor& xh_u) {
  Exl3Args a{};
  a.x = P<const __nv_bfloat16>(x);
  a.ldx = x.stride(0);
  a.suh_g = P<const __half>(suh_g);
  a.suh_u = P<const __half>(suh_u);
  a.K = (int)suh_g.size(-1);
  a.pair_token = P<const int>(pair_token);
  a.pair_expert = P<const int>(pair_expert);
  a.pairs = (int)pair_token.size(0);
  a.xh_g = P<__half>(xh_g);
  a.xh_u = P<__half>(xh_u);
  a.n_rows = x.size(0);
  a.n_experts = suh_g.size(0);
  TORCH_CHECK(xh_g.size(0) >= a.pairs && xh_u.size(0) >= a.pairs);
  check(g53_exl3_rot_in(a, stream()), "exl3_rot_in");
}

void moe_route_large(const Tensor& logits, const Tensor& bias, int64_t top_k, double scale, bool norm,
                     const Tensor& topk_ids, const Tensor& topk_w, const Tensor& group_count,
                     const Tensor& group_expert, const Tensor& group_offset, const Tensor& pair_token,
                     const Tensor& pair_expert, const Tensor& pair_w, const Tensor& pair_of, const Tensor& counts,
                     const Tensor& fill) {
  RouteArgs a{};
  a.logits = P<const float>(logits);
  a.bias = P<const float>(bias);
  a.R = (int)logits.size(0);
  a.E = (int)logits.size(1);
  a.top_k = (int)top_k;
  a.scale = (float)scale;
  a.norm = norm ? 1 : 0;
  a.topk_ids = P<int>(topk_ids);
  a.topk_w = P<float>(topk_w);
  a.group_count = P<int>(group_count);
  a.group_expert = P<int>(group_expert);
  a.group_offset = P<int>(group_offset);
  a.pair_token = P<int>(pair_token);
  a.pair_expert = P<int>(pair_expert);
  a.pair_w = P<float>(pair_w);
  a.pair_of = P<int>(pair_of);
  a.max_groups = (int)group_expert.size(0);
  TORCH_CHECK(counts.numel() >= a.E && fill.numel() >= a.E);
  check(g53_moe_route_large(a, P<int>(counts), P<int>(fill), stream()), "moe_route_large");
}

void moe_prefill(const Tensor& tr0, const OptT& tr1, const Tensor& svh0, const OptT& svh1, const OptT& suh_next,
                 const OptT& pair_w, const Tensor& group_count, const Tensor& group_expert, const Tensor& group_offset,
                 const Tensor& x0, const OptT& x1, const Tensor& out, double limit, bool gate_up) {
  MoePrefillArgs p{};
  p.tr0 = P<const int16_t>(tr0);
  p.tr1 = tr1.has_value() ? P<const int16_t>(tr1) : p.tr0;
  p.svh0 = P<const __half>(svh0);
  p.svh1 = P<const __half>(svh1);
  p.suh_next = P<const __half>(suh_next);
  p.pair_w = P<const float>(pair_w);
  p.group_count = P<const int>(group_count);
  p.group_expert = P<const int>(group_expert);
  p.group_offset = P<const int>(group_offset);
  p.n_experts = tr0.size(0);
  p.x0 = P<const __half>(x0);
  p.x1 = P<const __half>(x1);
  p.rows = x0.size(0);
  p.K = (int)x0.size(1);
  p.N = (int)svh0.size(-1);
  p.max_groups = (int)group_expert.size(0);
  p.out = out.data_ptr();
  p.limit = (float)limit;
  p.err = P<int>(err_word(x0));
  TORCH_CHECK(x0.scalar_type() == at::kHalf && x0.is_contiguous(), "activations must be contiguous f16");
  TORCH_CHECK(out.size(0) >= p.rows && out.size(1) == p.N, "out shape");
  check(g53_moe_prefill(p, gate_up, stream()), "moe_prefill");
}

// accumulate: 0 out = sum of the pair rows; 1 out += them (out first); 2 out = (sum of them) + out
void moe_combine(const Tensor& yd, const Tensor& pair_of, int64_t top_k, const Tensor& out, int64_t accumulate) {
  check(g53_moe_combine(P<const float>(yd), P<const int>(pair_of), (int)out.size(0), (int)top_k, (int)out.size(1),
                        P<float>(out), (int)accumulate, stream()),
        "moe_combine");
}

Tensor exl3_unpack(const Tensor& tr, int64_t K, int64_t N) {
  auto out = torch::empty({K, N}, tr.options().dtype(at::kHalf));
  check(g53_exl3_unpack(P<const int16_t>(tr), (int)K, (int)N, P<__half>(out), stream()), "exl3_unpack");
  return out;
}

// ------------------------------------------------------------------------------------------------- mHC / norms
// prefill-sized mHC launches use the tensor-core partial pass unless GLM53_TC_HC=0
static bool tc_hc_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = std::getenv("GLM53_TC_HC");
    v = (e && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

void hc_post_pre(const Tensor& X, const OptT& branch, const OptT& post, const OptT& comb, const OptT& fn,
                 const OptT& base, const OptT& hscale, const OptT& norm_w, const OptT& normed,
                 const OptT& post_out, const OptT& comb_out, const Tensor& part, double eps, double hc_eps,
                 int64_t iters, int64_t tensor_cores) {
  HcArgs a{};
  a.X = P<__nv_bfloat16>(X);
  a.branch = P<const float>(branch);
  a.post = P<const float>(post);
  a.comb = P<const float>(comb);
  a.fn = P<const __nv_bfloat16>(fn);
  a.base = P<const float>(base);
  a.hscale = P<const float>(hscale);
  a.norm_w = P<const __nv_bfloat16>(norm_w);
  a.normed = P<__nv_bfloat16>(normed);
  a.post_out = P<float>(post_out);
  a.comb_out = P<float>(comb_out);
  a.part = P<float>(part);
  a.R = (int)X.size(0);
  a.S = (int)X.size(1);
  a.D = (int)X.size(2);
  a.eps = (float)eps;
  a.hc_eps = (float)hc_eps;
  a.iters = (int)iters;
  TORCH_CHECK(X.is_contiguous(), "X must be contiguous [R, S, D]");
  a.gath = nullptr;
  a.use_tc = (tensor_cores < 0 ? tc_hc_enabled() : tensor_cores > 0) ? 1 : 0;
  a.err = P<int>(err_word(X));
  TORCH_CHECK(part.numel() >= (int64_t)a.R * (a.D / 64) * 32, "part scratch too small");
  check(g53_hc_post_pre(a, stream()), "hc_post_pre");
}

void embed(const Tensor& ids, const Tensor& table, const Tensor& X) {
  check(g53_embed(P<const int>(ids), P<const __nv_bfloat16>(table), (int)table.size(0), (int)X.size(0),
                  (int)X.size(2), (int)X.size(1), P<__nv_bfloat16>(X), stream()),
        "embed");
}

void stream_mean_norm(const Tensor& X, const Tensor& w, double eps, const OptT& hidden, const Tensor& normed) {
  check(g53_stream_mean_norm(P<const __nv_bfloat16>(X), (int)X.size(0), (int)X.size(1), (int)X.size(2),
                             P<const __nv_bfloat16>(w), (float)eps, P<__nv_bfloat16>(hidden),
                             P<__nv_bfloat16>(normed), stream()),
        "stream_mean_norm");
}

void rmsnorm(const Tensor& x, const Tensor& w, double eps, const Tensor& y) {
  TORCH_CHECK(x.stride(-1) == 1 && y.stride(-1) == 1);
  check(g53_rmsnorm(P<const __nv_bfloat16>(x), x.stride(0), P<const __nv_bfloat16>(w), (int)x.size(0),
                    (int)x.size(1), (float)eps, P<__nv_bfloat16>(y), y.stride(0), stream()),
        "rmsnorm");
}

void rmsnorm_f32(const Tensor& x, const Tensor& w, double eps, const Tensor& y) {
  TORCH_CHECK(x.is_contiguous() && y.is_contiguous() && x.scalar_type() == at::kFloat);
  check(g53_rmsnorm_f32(P<const float>(x), P<const __nv_bfloat16>(w), (int)x.size(0), (int)x.size(1), (float)eps,
                        P<__nv_bfloat16>(y), stream()),
        "rmsnorm_f32");
}

void block_attn(const Tensor& qkv, int64_t H, int64_t Dh, int64_t block, double scale, const Tensor& o) {
  TORCH_CHECK(qkv.is_contiguous() && o.is_contiguous());
  check(g53_block_attn(P<const __nv_bfloat16>(qkv), (int)qkv.size(0), (int)H, (int)Dh, (int)block, (float)scale,
                       P<__nv_bfloat16>(o), stream()),
        "block_attn");
}

// post (reducing the ranks' pushed partials in rank order) fused with pre
void hc_post_pre_tp(const Tensor& X, const Tensor& gath, int64_t slot, int64_t world, const Tensor& flags,
                    const Tensor& epoch, const Tensor& done, const Tensor& err, const Tensor& post,
                    const Tensor& comb, const OptT& fn, const OptT& base, const OptT& hscale, const OptT& norm_w,
                    const OptT& normed, const OptT& post_out, const OptT& comb_out, const Tensor& part, double eps,
                    double hc_eps, int64_t iters) {
  HcArgs a{};
  a.X = P<__nv_bfloat16>(X);
  a.post = P<const float>(post);
  a.comb = P<const float>(comb);
  a.fn = P<const __nv_bfloat16>(fn);
  a.base = P<const float>(base);
  a.hscale = P<const float>(hscale);
  a.norm_w = P<const __nv_bfloat16>(norm_w);
  a.normed = P<__nv_bfloat16>(normed);
  a.post_out = P<float>(post_out);
  a.comb_out = P<float>(comb_out);
  a.part = P<float>(part);
  a.R = (int)X.size(0);
  a.S = (int)X.size(1);
  a.D = (int)X.size(2);
  a.eps = (float)eps;
  a.hc_eps = (float)hc_eps;
  a.iters = (int)iters;
  a.gath = P<const float>(gath);
  a.gath_slot = slot;
  a.world = (int)world;
  a.flags = reinterpret_cast<const unsigned*>(flags.data_ptr());
  a.epoch = reinterpret_cast<unsigned*>(epoch.data_ptr());
  a.done = reinterpret_cast<unsigned*>(done.data_ptr());
  a.err = P<int>(err);
  TORCH_CHECK(X.is_contiguous());
  check(g53_hc_post_pre(a, stream()), "hc_post_pre_tp");
}

// ------------------------------------------------------------------------------------------------- KDA
// seq: int32 [5, B] device tensor: rows row0, nrows, state-in index, state-out index, conv slot
KdaArgs kda_args(const Tensor& proj, const Tensor& seq, int64_t max_rows, int64_t H, int64_t Dh, int64_t taps) {
  KdaArgs a{};
  a.proj = P<const __nv_bfloat16>(proj);
  a.ldp = proj.stride(0);
  TORCH_CHECK(seq.scalar_type() == at::kInt && seq.dim() == 2 && seq.size(0) == 5 && seq.stride(1) == 1,
              "seq must be int32 [5, B] (rows contiguous)");
  const int B = (int)seq.size(1);
  const int64_t ld = seq.stride(0);
  const int* s = P<const int>(seq);
  a.row0 = s; a.nrows = s + ld; a.s_in = s + 2 * ld; a.s_out = s + 3 * ld; a.conv_slot = s + 4 * ld;
  a.B = B;
  a.max_rows = (int)max_rows;
  a.R = (int)proj.size(0);
  a.H = (int)H; a.Dh = (int)Dh; a.taps = (int)taps;
  return a;
}

void kda_conv(const Tensor& proj, const Tensor& seq, int64_t max_rows, const Tensor& conv_w, const Tensor& conv_pool,
              const Tensor& qkv, int64_t H, int64_t Dh) {
  KdaArgs a = kda_args(proj, seq, max_rows, H, Dh, conv_w.size(1));
  a.conv_w = P<const float>(conv_w);
  a.conv_pool = P<__nv_bfloat16>(conv_pool);
  a.n_conv = conv_pool.size(0);
  a.qkv = P<__nv_bfloat16>(qkv);
  check(g53_kda_conv(a, stream()), "kda_conv");
}

void kda_conv_commit(const Tensor& proj, const Tensor& seq, const Tensor& conv_pool, int64_t H, int64_t Dh,
                     int64_t taps) {
  KdaArgs a = kda_args(proj, seq, 0, H, Dh, taps);
  a.conv_pool = P<__nv_bfloat16>(conv_pool);
  a.n_conv = conv_pool.size(0);
  check(g53_kda_conv_commit(a, stream()), "kda_conv_commit");
}

void kda_recurrent(const Tensor& proj, const Tensor& seq, const Tensor& f, const Tensor& qkv, const Tensor& a_log,
                   const Tensor& dt_bias, const Tensor& S_pool, const OptT& o_raw, int64_t H, int64_t Dh,
                   int64_t b_off, double lower) {
  KdaArgs a = kda_args(proj, seq, 0, H, Dh, 0);
  a.f = P<const __nv_bfloat16>(f);
  a.qkv = P<__nv_bfloat16>(qkv);
  a.a_log = P<const float>(a_log);
  a.dt_bias = P<const float>(dt_bias);
  a.S_pool = P<float>(S_pool);
  a.n_states = S_pool.size(0);
  a.o_raw = P<float>(o_raw);
  a.b_off = (int)b_off;
  a.lower = (float)lower;
  check(g53_kda_recurrent(a, stream()), "kda_recurrent");
}

// fused decode window (rows per sequence <= 16, Dh 128, 4 taps): f_b / g_b from the f_a / g_a columns of proj,
// conv (qkv and f stored for the commit replay), recurrence S_in -> S_out, gated norm into out
void kda_decode(const Tensor& proj, const Tensor& seq, int64_t max_rows, const Tensor& fb_w, const Tensor& fb_s,
                const Tensor& gb_w, const Tensor& gb_s, const Tensor& conv_w, const Tensor& conv_pool,
                const Tensor& qkv, const Tensor& f_store, const Tensor& a_log, const Tensor& dt_bias,
                const Tensor& o_norm, const Tensor& S_pool, const Tensor& out, int64_t H, int64_t Dh, int64_t fa_off,
                int64_t b_off, double lower, double eps) {
  KdaArgs a = kda_args(proj, seq, max_rows, H, Dh, conv_w.size(1));
  TORCH_CHECK(fb_w.is_contiguous() && gb_w.is_contiguous() && fb_w.size(0) == H * Dh && fb_w.size(1) == Dh &&
              gb_w.sizes() == fb_w.sizes(), "kda_decode: f_b / g_b must be [H*Dh, Dh] contiguous");
  TORCH_CHECK(qkv.stride(0) == 3 * H * Dh && f_store.stride(0) == H * Dh && out.stride(0) == H * Dh,
              "kda_decode: qkv / f / out rows must be dense");
  a.fb_w = P<const uint8_t>(fb_w); a.fb_s = P<const float>(fb_s);
  a.gb_w = P<const uint8_t>(gb_w); a.gb_s = P<const float>(gb_s);
  a.conv_w = P<const float>(conv_w);
  a.conv_pool = P<__nv_bfloat16>(conv_pool);
  a.n_conv = conv_pool.size(0);
  a.qkv = P<__nv_bfloat16>(qkv);
  a.f_store = P<__nv_bfloat16>(f_store);
  a.a_log = P<const float>(a_log);
  a.dt_bias = P<const float>(dt_bias);
  a.o_norm = P<const __nv_bfloat16>(o_norm);
  a.S_pool = P<float>(S_pool);
  a.n_states = S_pool.size(0);
  a.out = P<__nv_bfloat16>(out);
  a.fa_off = (int)fa_off;
  a.b_off = (int)b_off;
  a.lower = (float)lower;
  a.eps = (float)eps;
  TORCH_CHECK(g53_kda_decode_ok(a), "kda_decode: unsupported shape or alignment");
  check(g53_kda_decode(a, stream()), "kda_decode");
}

void kda_chunk(const Tensor& proj, const Tensor& seq, const Tensor& f, const Tensor& qkv, const Tensor& a_log,
               const Tensor& dt_bias, const Tensor& S_pool, const Tensor& o_raw, int64_t H, int64_t Dh, int64_t b_off,
               double lower, const Tensor& scratch) {
  KdaArgs a = kda_args(proj, seq, 0, H, Dh, 0);
  TORCH_CHECK(scratch.scalar_type() == at::kFloat && scratch.is_contiguous(), "kda_chunk scratch must be fp32");
  const int64_t per_slot = g53_kda_chunk_scratch_floats(64, 0, (int)H, (int)Dh) / 2;   // one slot, all heads
  a.scr = P<float>(scratch);
  a.scr_slots = (int)(scratch.numel() / per_slot);
  a.f = P<const __nv_bfloat16>(f);
  a.qkv = P<__nv_bfloat16>(qkv);
  a.a_log = P<const float>(a_log);
  a.dt_bias = P<const float>(dt_bias);
  a.S_pool = P<float>(S_pool);
  a.n_states = S_pool.size(0);
  a.o_raw = P<float>(o_raw);
  a.b_off = (int)b_off;
  a.lower = (float)lower;
  check(g53_kda_chunk(a, stream()), "kda_chunk");
}

void kda_gated_norm(const Tensor& o_raw, const Tensor& gate, const Tensor& o_norm, const Tensor& out, int64_t H,
                    int64_t Dh, double eps) {
  KdaArgs a{};
  a.o_raw = P<float>(o_raw);
  a.gate = P<const __nv_bfloat16>(gate);
  a.o_norm = P<const __nv_bfloat16>(o_norm);
  a.out = P<__nv_bfloat16>(out);
  a.R = (int)out.size(0);
  a.H = (int)H; a.Dh = (int)Dh; a.eps = (float)eps;
  check(g53_kda_gated_norm(a, stream()), "kda_gated_norm");
}

// ------------------------------------------------------------------------------------------------- MLA / DSA
void mla_prep(const Tensor& qkv_a, const Tensor& q_norm, const Tensor& kv_norm, const Tensor& qr,
              const Tensor& kv_cache, const Tensor& kv_scale, const OptT& kpe_cache, const Tensor& slots,
              const Tensor& positions, int64_t q_lora, int64_t kv_lora, int64_t rope, double eps, double theta) {
  MlaPrepArgs a{};
  a.qkv_a = P<const __nv_bfloat16>(qkv_a);
  a.ld = qkv_a.stride(0);
  a.q_norm = P<const __nv_bfloat16>(q_norm);
  a.kv_norm = P<const __nv_bfloat16>(kv_norm);
  a.qr = P<__nv_bfloat16>(qr);
  a.kv_cache = P<uint8_t>(kv_cache);
  a.kv_scale = P<float>(kv_scale);
  a.kpe_cache = P<__nv_bfloat16>(kpe_cache);
  a.slots = P<const int>(slots);
  a.positions = P<const int>(positions);
  a.R = (int)qkv_a.size(0);
  a.q_lora = (int)q_lora; a.kv_lora = (int)kv_lora; a.rope = (int)rope;
  a.eps = (float)eps; a.theta = (float)theta;
  a.n_slots = kv_cache.size(0);
  check(g53_mla_prep(a, stream()), "mla_prep");
}

void rope_q(const Tensor& q, const Tensor& positions, int64_t nope, int64_t rope, double theta) {
  TORCH_CHECK(q.is_contiguous() && q.dim() == 3);
  check(g53_rope_q(P<__nv_bfloat16>(q), (int)q.size(0), (int)q.size(1), (int)q.size(2), (int)nope, (int)rope,
                   P<const int>(positions), (float)theta, stream()),
        "rope_q");
}

// the tensor-core sparse MLA kernel is used (where its shape applies) unless GLM53_TC_MLA=0
static bool tc_mla_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = std::getenv("GLM53_TC_MLA");
    v = (e && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}
static bool mla_tc_shape(const MlaAttnArgs& a) { return a.L == 512 && a.rope == 0 && a.H >= 1 && a.H <= 64; }

// tensor_cores: -1 default (GLM53_TC_MLA), 0 CUDA-core kernel, 1 tensor-core kernel (error if the shape does not fit)
void mla_decode(const Tensor& q_lat, const OptT& q_pe, int64_t q_pe_ld, int64_t q_pe_hs, const Tensor& kv_cache,
                const Tensor& kv_scale, const OptT& kpe_cache, const Tensor& sel, const Tensor& sel_count,
                int64_t rope, double sm_scale, int64_t splits, const Tensor& part_o, const Tensor& part_ml,
                const Tensor& o_lat, int64_t tensor_cores) {
  MlaAttnArgs a{};
  a.q_lat = P<const __nv_bfloat16>(q_lat);
  a.q_pe = P<const __nv_bfloat16>(q_pe);
  a.q_pe_ld = q_pe_ld;
  a.q_pe_hs = (int)q_pe_hs;
  a.kv_cache = P<const uint8_t>(kv_cache);
  a.kv_scale = P<const float>(kv_scale);
  a.kpe_cache = P<const __nv_bfloat16>(kpe_cache);
  a.n_slots = kv_cache.size(0);
  a.sel = P<const int>(sel);
  a.sel_count = P<const int>(sel_count);
  a.max_sel = (int)sel.size(1);
  a.R = (int)q_lat.size(0);
  a.H = (int)q_lat.size(1);
  a.L = (int)q_lat.size(2);
  a.rope = (int)rope;
  a.sm_scale = (float)sm_scale;
  a.splits = (int)splits;
  a.part_o = P<float>(part_o);
  a.part_ml = P<float>(part_ml);
  a.o_lat = P<__nv_bfloat16>(o_lat);
  a.use_tc = (tensor_cores < 0 ? tc_mla_enabled() : tensor_cores > 0) && mla_tc_shape(a) ? 1 : 0;
  TORCH_CHECK(tensor_cores <= 0 || a.use_tc, "tensor-core MLA needs L = 512, no rope and at most 64 heads");
  // split partials (the CUDA-core kernel stages every row's partials, the tensor-core kernel only split rows)
  if (!a.use_tc || a.splits > 1) {
    TORCH_CHECK(part_o.numel() >= (int64_t)a.R * a.splits * a.H * a.L, "part_o too small");
    TORCH_CHECK(part_ml.numel() >= (int64_t)a.R * a.splits * a.H * 2, "part_ml too small");
  }
  a.err = P<int>(err_word(q_lat));
  check(g53_mla_decode(a, stream()), "mla_decode");
}

DsaArgs dsa_args(const Tensor& iproj, const Tensor& ln_w, const Tensor& ln_b, const Tensor& ape, const OptT& qi,
                 const Tensor& ik_cache, const Tensor& ig_cache, const Tensor& pool_cache, const Tensor& pool_scale,
                 const Tensor& slots, const Tensor& positions, const Tensor& block_table, const Tensor& row_seq,
                 int64_t block_size, int64_t IH, int64_t kpool, int64_t topk_pools, double eps, const OptT& logits,
                 const OptT& sel, const OptT& sel_count) {
  DsaArgs a{};
  a.iproj = P<const float>(iproj);
  a.ldi = iproj.stride(0);
  a.ln_w = P<const float>(ln_w);
  a.ln_b = P<const float>(ln_b);
  a.ape = P<const float>(ape);
  a.qi = P<const __nv_bfloat16>(qi);
  a.ik_cache = P<__nv_bfloat16>(ik_cache);
  a.ig_cache = P<float>(ig_cache);
  a.pool_cache = P<uint8_t>(pool_cache);
  a.pool_scale = P<float>(pool_scale);
  a.n_pools = pool_scale.size(0);
  a.slots = P<const int>(slots);
  a.positions = P<const int>(positions);
  a.block_table = P<const int>(block_table);
  a.row_seq = P<const int>(row_seq);
  a.bt_ld = block_table.dim() == 2 ? (int)block_table.stride(0) : 0;
  a.block_size = (int)block_size;
  a.R = (int)iproj.size(0);
  a.IH = (int)IH;
  a.ID = (int)ln_w.size(0);
  a.kpool = (int)kpool;
  a.topk_pools = (int)topk_pools;
  a.eps = (float)eps;
  a.logits = P<float>(logits);
  a.max_pools = (logits.has_value() && logits->defined()) ? (int)logits->size(1) : 0;
  a.sel = P<int>(sel);
  a.sel_count = P<int>(sel_count);
  a.max_sel = (sel.has_value() && sel->defined()) ? (int)sel->size(1) : 0;
  return a;
}

// ik_rows / ig_rows: [>= R, ID] row buffers of this launch; ik_ring / ig_ring: [state slots * ring, ID] tail rings;
// seq_desc: [5, sequences] int32 (row0, nrows, s_in, s_out, state slot) of the launch
void dsa_update(const Tensor& iproj, const Tensor& ln_w, const Tensor& ln_b, const Tensor& ape,
                const Tensor& ik_rows, const Tensor& ig_rows, const Tensor& ik_ring, const Tensor& ig_ring,
                const Tensor& pool_cache, const Tensor& pool_scale, const Tensor& slots, const Tensor& positions,
                const Tensor& block_table, const Tensor& row_seq, const Tensor& seq_desc, int64_t block_size,
                int64_t IH, int64_t kpool, double eps) {
  DsaArgs a = dsa_args(iproj, ln_w, ln_b, ape, {}, ik_rows, ig_rows, pool_cache, pool_scale, slots, positions,
                       block_table, row_seq, block_size, IH, kpool, 0, eps, {}, {}, {});
  TORCH_CHECK(ik_rows.size(0) >= a.R && ig_rows.size(0) >= a.R, "dsa_update: row buffers too small");
  TORCH_CHECK(ik_ring.size(0) % kDsaRing == 0 && ig_ring.size(0) == ik_ring.size(0), "dsa_update: ring shape");
  TORCH_CHECK(seq_desc.dim() == 2 && seq_desc.size(0) == 5 && seq_desc.scalar_type() == at::kInt, "seq_desc");
  a.ik_ring = P<__nv_bfloat16>(ik_ring);
  a.ig_ring = P<float>(ig_ring);
  a.n_owners = ik_ring.size(0) / kDsaRing;
  a.seq_desc = P<const int>(seq_desc);
  a.seq_ld = (int)seq_desc.stride(0);
  check(g53_dsa_update(a, stream()), "dsa_update");
}

// the tcgen05 indexer logits are used unless GLM53_TC_DSA=0
static bool tc_dsa_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = std::getenv("GLM53_TC_DSA");
    v = (e && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

// logits only (tests and benchmarks): tensor-core or CUDA-core kernel
void dsa_logits(const Tensor& iproj, const Tensor& qi, const Tensor& ln_w, const Tensor& pool_cache,
                const Tensor& pool_scale, const Tensor& positions, const Tensor& block_table, const Tensor& row_seq,
                int64_t block_size, int64_t IH, int64_t kpool, const Tensor& logits, bool tensor_cores) {
  DsaArgs a = dsa_args(iproj, ln_w, ln_w, ln_w, qi, pool_cache, pool_scale, pool_cache, pool_scale, positions,
                       positions, block_table, row_seq, block_size, IH, kpool, 0, 0, logits, {}, {});
  a.ik_cache = nullptr;
  a.ig_cache = nullptr;
  a.err = P<int>(err_word(logits));
  if (tensor_cores) check(g53_dsa_logits_tc(a, stream()), "dsa_logits_tc");
  else check(g53_dsa_logits(a, stream()), "dsa_logits");
}

void dsa_select(const Tensor& iproj, const Tensor& qi, const Tensor& ln_w, const Tensor& pool_cache,
                const Tensor& pool_scale, const Tensor& positions, const Tensor& block_table, const Tensor& row_seq,
                int64_t block_size, int64_t IH, int64_t kpool, int64_t topk_pools, const Tensor& logits,
                const Tensor& sel, const Tensor& sel_count) {
  DsaArgs a = dsa_args(iproj, ln_w, ln_w, ln_w, qi, pool_cache, pool_scale, pool_cache, pool_scale, positions,
                       positions, block_table, row_seq, block_size, IH, kpool, topk_pools, 0, logits, sel, sel_count);
  a.ik_cache = nullptr;
  a.ig_cache = nullptr;
  a.err = P<int>(err_word(logits));
  // tcgen05 logits for prefill-sized launches where the head count fits the kernel (IH | 32, ID = 128).  Decode
  // windows (a few rows: one query tile, pools split over CTAs) launch both kernels: the CUDA-core kernel is
  // faster up to kDsaTcMinPools complete pools (measured at 8 rows: 37 vs 47 us at 8192 pools), the tcgen05 kernel
  // above (76 vs 108 us at 32768 pools, 94 vs 403 us at 131072); the device picks from the rows' positions
  constexpr int kDsaTcMinPools = 16384;
  const bool tc_ok = tc_dsa_enabled() && a.ID == 128 && (a.IH == 4 || a.IH == 8 || a.IH == 16 || a.IH == 32);
  if (tc_ok && a.R >= 64) {
    check(g53_dsa_logits_tc(a, stream()), "dsa_logits_tc");
  } else if (tc_ok && a.max_pools > kDsaTcMinPools) {
    a.tc_min_pools = kDsaTcMinPools;
    check(g53_dsa_logits(a, stream()), "dsa_logits");
    check(g53_dsa_logits_tc(a, stream()), "dsa_logits_tc");
    a.tc_min_pools = 0;
  } else {
    check(g53_dsa_logits(a, stream()), "dsa_logits");
  }
  check(g53_dsa_select(a, stream()), "dsa_select");
}

// ------------------------------------------------------------------------------------------------- sampling
void argmax_rows(const Tensor& logits, int64_t vocab_offset, const Tensor& best_val, const Tensor& best_id) {
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.stride(-1) == 1);
  check(g53_argmax_rows(P<const float>(logits), (int)logits.size(0), (int)logits.size(1), logits.stride(0),
                        (int)vocab_offset, P<float>(best_val), P<int>(best_id), stream()),
        "argmax_rows");
}

void greedy_verify(const Tensor& draft, const Tensor& target, bool forced, const Tensor& accepted,
                   const Tensor& next_tokens) {
  VerifyArgs a{};
  a.draft = P<const int>(draft);
  a.target_argmax = P<const int>(target);
  a.B = (int)draft.size(0);
  a.K = (int)draft.size(1);
  a.forced = forced ? 1 : 0;
  a.accepted = P<int>(accepted);
  a.next_tokens = P<int>(next_tokens);
  check(g53_greedy_verify(a, stream()), "greedy_verify");
}

void rejection_sample(const Tensor& target_probs, const Tensor& draft_probs, const Tensor& draft, int64_t seed,
                      const Tensor& positions, bool block, const Tensor& accepted, const Tensor& next_tokens,
                      const OptT& scratch) {
  RejectArgs a{};
  a.target_probs = P<const float>(target_probs);
  a.draft_probs = P<const float>(draft_probs);
  a.draft = P<const int>(draft);
  a.B = (int)draft.size(0);
  a.K = (int)draft.size(1);
  a.V = (int)target_probs.size(2);
  a.seed = (uint64_t)seed;
  a.positions = P<const int64_t>(positions);
  a.block = block ? 1 : 0;
  a.accepted = P<int>(accepted);
  a.next_tokens = P<int>(next_tokens);
  a.scratch = P<float>(scratch);
  check(g53_rejection_sample(a, stream()), "rejection_sample");
}

}  // namespace

void register_exl3_codec(pybind11::module& m);   // exl3_codec.cpp (host codec)

namespace {
// (enabled, [(code, index, limit, count), ...]) of the bounds-checked build's records that saw an error
py::tuple bounds_status() {
  py::list out;
  std::lock_guard<std::mutex> lock(g53_bounds_mu);
  for (const void* sym : g53_bounds_symbols()) {
    G53BoundsRecHost r{};
    const cudaError_t e = cudaMemcpyFromSymbol(&r, sym, sizeof(r));
    TORCH_CHECK(e == cudaSuccess, "bounds_status: ", cudaGetErrorString(e));
    if (r.count) out.append(py::make_tuple(r.code, r.index, r.limit, r.count));
  }
  return py::make_tuple(!g53_bounds_symbols().empty(), out);
}

void bounds_reset() {
  std::lock_guard<std::mutex> lock(g53_bounds_mu);
  const G53BoundsRecHost z{};
  for (const void* sym : g53_bounds_symbols()) {
    const cudaError_t e = cudaMemcpyToSymbol(sym, &z, sizeof(z));
    TORCH_CHECK(e == cudaSuccess, "bounds_reset: ", cudaGetErrorString(e));
  }
}
}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  register_exl3_codec(m);
  m.doc() = "glm53 sm_100a kernels";
  m.def("gemv", &gemv, py::arg("x"), py::arg("w"), py::arg("scale"), py::arg("y"), py::arg("mode"), py::arg("limit"),
        py::arg("ks") = 0, py::arg("cl") = 0);
  m.def("gemm_w8", &gemm_w8);
  m.def("quant_rows", &quant_rows);
  m.def("gemm_w8q", &gemm_w8q);
  m.def("gemm_bf16", &gemm_bf16);
  m.def("gemm_w8a16", &gemm_w8a16);
  m.def("gemm_error", &gemm_error);
  m.def("l2_prefetch", &l2_prefetch, py::arg("tensors"), py::arg("max_bytes"));
  m.def("gemm_w8a16_push", &gemm_w8a16_push);
  m.def("gemm_ag_w8a16", &gemm_ag_w8a16);
  m.def("signal_peers", &signal_peers);
  m.def("moe_route", &moe_route);
  m.def("exl3_moe", &exl3_moe, py::arg("x"), py::arg("tr_g"), py::arg("suh_g"), py::arg("svh_g"), py::arg("tr_u"),
        py::arg("suh_u"), py::arg("svh_u"), py::arg("tr_d"), py::arg("suh_d"), py::arg("svh_d"),
        py::arg("group_count"), py::arg("group_expert"), py::arg("group_offset"), py::arg("pair_token"),
        py::arg("pair_expert"), py::arg("pair_w"), py::arg("xh_g"), py::arg("xh_u"), py::arg("xd"), py::arg("yd"),
        py::arg("limit"), py::arg("prefetch") = std::vector<Tensor>{}, py::arg("prefetch_bytes") = 0);
  m.def("moe_combine", &moe_combine);
  m.def("moe_route_large", &moe_route_large);
  m.def("moe_prefill", &moe_prefill);
  m.def("exl3_rot_in", &exl3_rot_in);
  m.def("ep_moe_step", &ep_moe_step);
  m.def("bounds_status", &bounds_status);
  m.def("bounds_reset", &bounds_reset);
  m.def("exl3_unpack", &exl3_unpack);
  m.def("hc_post_pre", &hc_post_pre, py::arg("X"), py::arg("branch"), py::arg("post"), py::arg("comb"), py::arg("fn"),
        py::arg("base"), py::arg("hscale"), py::arg("norm_w"), py::arg("normed"), py::arg("post_out"),
        py::arg("comb_out"), py::arg("part"), py::arg("eps"), py::arg("hc_eps"), py::arg("iters"),
        py::arg("tensor_cores") = -1);
  m.def("hc_post_pre_tp", &hc_post_pre_tp);
  m.def("gemv_push", &gemv_push);
  m.def("embed", &embed);
  m.def("stream_mean_norm", &stream_mean_norm);
  m.def("rmsnorm", &rmsnorm);
  m.def("rmsnorm_f32", &rmsnorm_f32);
  m.def("block_attn", &block_attn);
  m.def("kda_conv", &kda_conv);
  m.def("kda_conv_commit", &kda_conv_commit);
  m.def("kda_recurrent", &kda_recurrent);
  m.def("kda_gated_norm", &kda_gated_norm);
  m.def("kda_chunk", &kda_chunk);
  m.def("dsa_logits", &dsa_logits);
  m.def("kda_chunk_scratch_floats", [](int64_t max_rows, int64_t max_seqs, int64_t H, int64_t Dh) {
    return g53_kda_chunk_scratch_floats((int)max_rows, (int)max_seqs, (int)H, (int)Dh);
  });
  m.def("mla_prep", &mla_prep);
  m.def("rope_q", &rope_q);
  m.def("mla_decode", &mla_decode, py::arg("q_lat"), py::arg("q_pe"), py::arg("q_pe_ld"), py::arg("q_pe_hs"),
        py::arg("kv_cache"), py::arg("kv_scale"), py::arg("kpe_cache"), py::arg("sel"), py::arg("sel_count"),
        py::arg("rope"), py::arg("sm_scale"), py::arg("splits"), py::arg("part_o"), py::arg("part_ml"),
        py::arg("o_lat"), py::arg("tensor_cores") = -1);
  m.def("kda_decode", &kda_decode);
  m.def("dconv", &dconv);
  m.def("dsa_update", &dsa_update);
  m.def("dsa_ring_positions", []() { return (int64_t)kDsaRing; });
  m.def("dsa_select", &dsa_select);
  m.def("argmax_rows", &argmax_rows);
  m.def("greedy_verify", &greedy_verify);
  m.def("rejection_sample", &rejection_sample);
  m.attr("GEMV_BF16") = (int)GEMV_BF16;
  m.attr("GEMV_F32") = (int)GEMV_F32;
  m.attr("GEMV_F32_ACC") = (int)GEMV_F32_ACC;
  m.attr("GEMV_SWIGLU") = (int)GEMV_SWIGLU;
}
