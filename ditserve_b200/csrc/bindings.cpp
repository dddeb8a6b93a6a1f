// torch bindings of the sm_100a kernels (module ditserve_b200._C).
// Thin: validate tensors, fill the launch structs from kernels.h, launch on
// the current CUDA stream.  All shape/stride rules are enforced here so a bad
// call raises a Python exception instead of reaching the GPU.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAException.h>

#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <tuple>

#include "kernels.h"

namespace {

void check_cuda_bf16_2d(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.scalar_type() == at::kBFloat16, name, " must be bfloat16");
  TORCH_CHECK(t.dim() == 2, name, " must be 2-D");
  TORCH_CHECK(t.stride(1) == 1, name, " must have unit column stride");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0, name, " must be 16-byte aligned");
}

const void* opt_ptr(const c10::optional<at::Tensor>& t) { return t.has_value() ? t->data_ptr() : nullptr; }

// Tail split of the attention grid.  With U (query block, head, batch) units of 256 rows over
// S SMs (one CTA each), the last round holds U mod S units and leaves the rest of the GPU
// idle.  Those tail units are cut into k key ranges (k chosen to fill the last round best),
// their parts run after the whole units and attention_merge combines them.  The work list and
// the merge table depend only on the shape, so they are built once per (device, shape).
struct SplitPlan {
  at::Tensor work;    // int32 [num_work, 4] on the device
  at::Tensor merge;   // int32 [num_merge, 4] on the device
  int num_work = 0, num_merge = 0, slots = 0;
};

// Number of key ranges for the tail units (1: no split): the k in 2..8 (each range at least 8
// key tiles) that minimises full + ceil(tail * k / sms) / k, kept only when it saves 3 %.
int tail_split_parts(int64_t units, int64_t tiles, int64_t sms) {
  if (sms <= 0) return 1;
  const int64_t full = units / sms, tail = units - full * sms;
  int best_k = 1;
  double best_t = static_cast<double>(full + 1);
  for (int k = 2; k <= 8 && tail > 0 && tiles / k >= 8; ++k) {
    const double t = full + static_cast<double>((tail * k + sms - 1) / sms) / k;
    if (t < best_t * 0.97) {
      best_t = t;
      best_k = k;
    }
  }
  return best_k;
}

const SplitPlan* split_plan(int64_t batch, int64_t seq_q, int64_t seq_k, int64_t heads, const at::Device& dev) {
  static const bool enabled = [] {
    const char* e = std::getenv("DS_ATTN_SPLIT");
    return e == nullptr || std::atoi(e) != 0;
  }();
  if (!enabled) return nullptr;
  static std::mutex mu;
  static std::map<std::tuple<int, int64_t, int64_t, int64_t, int64_t>, std::unique_ptr<SplitPlan>> cache;
  const auto key = std::make_tuple(static_cast<int>(dev.index()), batch, seq_q, seq_k, heads);
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second.get();
  std::unique_ptr<SplitPlan> plan;
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev.index());
  const int64_t nq = (seq_q + 255) / 256, tiles = (seq_k + 127) / 128, units = nq * heads * batch;
  const int64_t tail = sms > 0 ? units % sms : 0;
  const int best_k = tail_split_parts(units, tiles, sms);
  if (best_k > 1 && units < (1 << 16) && tiles < (1 << 16)) {
    plan = std::make_unique<SplitPlan>();
    std::vector<int32_t> work, merge;
    const int64_t whole = units - tail;
    auto unit_of = [&](int64_t u, int32_t& qb, int32_t& h, int32_t& b) {
      qb = static_cast<int32_t>(u % nq);
      h = static_cast<int32_t>((u / nq) % heads);
      b = static_cast<int32_t>(u / (nq * heads));
    };
    for (int64_t u = 0; u < whole; ++u) {
      int32_t qb, h, b;
      unit_of(u, qb, h, b);
      work.insert(work.end(), {qb, h, b, static_cast<int32_t>(0 | (tiles << 16))});
    }
    int32_t slot = 0;
    for (int64_t u = whole; u < units; ++u) {
      int32_t qb, h, b;
      unit_of(u, qb, h, b);
      merge.insert(merge.end(), {qb, h, b, static_cast<int32_t>(slot | (best_k << 16))});
      for (int i = 0; i < best_k; ++i) {
        const int32_t t0 = static_cast<int32_t>(tiles * i / best_k), t1 = static_cast<int32_t>(tiles * (i + 1) / best_k);
        work.insert(work.end(), {static_cast<int32_t>(qb | ((slot + 1) << 16)), h, b, static_cast<int32_t>(t0 | (t1 << 16))});
        ++slot;
      }
    }
    auto opts = at::TensorOptions().dtype(at::kInt);
    plan->num_work = static_cast<int>(work.size() / 4);
    plan->num_merge = static_cast<int>(merge.size() / 4);
    plan->slots = slot;
    plan->work = at::from_blob(work.data(), {plan->num_work, 4}, opts).clone().to(dev);
    plan->merge = at::from_blob(merge.data(), {plan->num_merge, 4}, opts).clone().to(dev);
  }
  const SplitPlan* out = plan.get();
  cache.emplace(key, std::move(plan));
  return out;
}

// Fills the work-list fields of `a` for a uniform one-source call when a split pays; the
// partial buffers come from the caching allocator and live until the launch is enqueued
// (stream-ordered reuse keeps them valid for the kernels that use them).
void apply_split(ds::AttnArgs& a, const at::Device& dev, std::vector<at::Tensor>& keep) {
  if (a.kv_sources != 1 || a.head_dim != 128) return;
  const SplitPlan* plan = split_plan(a.batch, a.seq_q, a.seq_k, a.heads, dev);
  if (plan == nullptr) return;
  auto f = at::TensorOptions().dtype(at::kFloat).device(dev);
  keep.push_back(at::empty({static_cast<int64_t>(plan->slots) * 256 * a.head_dim}, f));
  keep.push_back(at::empty({static_cast<int64_t>(plan->slots) * 256 * 2}, f));
  a.part_o = keep[keep.size() - 2].data_ptr<float>();
  a.part_ml = keep.back().data_ptr<float>();
  a.work = reinterpret_cast<const int4*>(plan->work.data_ptr<int32_t>());
  a.num_work = plan->num_work;
  a.merge_units = reinterpret_cast<const int4*>(plan->merge.data_ptr<int32_t>());
  a.num_merge_units = plan->num_merge;
}

int* status_ptr(const at::Tensor& status) {
  TORCH_CHECK(status.is_cuda() && status.scalar_type() == at::kInt && status.numel() >= 2,
              "status must be a CUDA int32 tensor with >= 2 elements");
  return status.data_ptr<int>();
}

void gemm(const at::Tensor& A, const at::Tensor& B, at::Tensor& C, const c10::optional<at::Tensor>& bias,
          int64_t epilogue, const c10::optional<at::Tensor>& R, const c10::optional<at::Tensor>& gate,
          int64_t gate_stride, int64_t rows_per_batch, const at::Tensor& status, int64_t bn_override,
          const c10::optional<at::Tensor>& row_batch, int64_t cta_pair) {
  check_cuda_bf16_2d(A, "A");
  check_cuda_bf16_2d(B, "B");
  check_cuda_bf16_2d(C, "C");
  TORCH_CHECK(A.size(1) == B.size(1), "gemm: K mismatch");
  TORCH_CHECK(C.size(0) == A.size(0) && C.size(1) == B.size(0), "gemm: C shape mismatch");
  if (bias.has_value()) {
    TORCH_CHECK(bias->is_contiguous() && bias->scalar_type() == at::kBFloat16 && bias->numel() == B.size(0),
                "gemm: bias must be contiguous bf16 [N]");
  }
  if (R.has_value()) {
    check_cuda_bf16_2d(*R, "R");
    TORCH_CHECK(R->size(0) == C.size(0) && R->size(1) == C.size(1), "gemm: residual shape mismatch");
  }
  if (gate.has_value()) {
    TORCH_CHECK(gate->is_cuda() && gate->scalar_type() == at::kFloat, "gemm: gate must be fp32 CUDA");
  }
  const c10::cuda::CUDAGuard guard(A.device());
  ds::GemmArgs a;
  a.A = A.data_ptr();
  a.lda = A.stride(0);
  a.B = B.data_ptr();
  a.ldb = B.stride(0);
  a.C = C.data_ptr();
  a.ldc = C.stride(0);
  a.M = static_cast<int>(A.size(0));
  a.N = static_cast<int>(B.size(0));
  a.K = static_cast<int>(A.size(1));
  a.bias = opt_ptr(bias);
  a.epilogue = static_cast<int>(epilogue);
  a.R = opt_ptr(R);
  a.ldr = R.has_value() ? R->stride(0) : 0;
  a.gate = gate.has_value() ? gate->data_ptr<float>() : nullptr;
  a.gate_stride = gate_stride;
  a.rows_per_batch = static_cast<int>(rows_per_batch);
  a.status = status_ptr(status);
  a.bn_override = static_cast<int>(bn_override);
  a.cta_pair = static_cast<int>(cta_pair);
  if (row_batch.has_value()) {
    TORCH_CHECK(row_batch->scalar_type() == at::kInt && row_batch->numel() >= A.size(0) && row_batch->is_cuda(),
                "gemm: row_batch must be int32 CUDA with one entry per row");
    a.row_batch = row_batch->data_ptr<int>();
  }
  ds::launch_gemm(a, at::cuda::getCurrentCUDAStream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();  // a failed launch raises here, never passes silently
}

void attention(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, at::Tensor& o,
               const c10::optional<at::Tensor>& lse, int64_t batch, int64_t seq_q, int64_t seq_k,
               const c10::optional<at::Tensor>& cu_q, const c10::optional<at::Tensor>& cu_k, int64_t max_seq_q,
               int64_t heads, int64_t heads_kv, int64_t head_dim, double scale, const at::Tensor& status,
               const c10::optional<at::Tensor>& seg, int64_t max_q_blocks, std::vector<at::Tensor> k_extra,
               std::vector<at::Tensor> v_extra, const c10::optional<at::Tensor>& blk_offsets,
               const c10::optional<at::Tensor>& blk_index) {
  check_cuda_bf16_2d(q, "q");
  check_cuda_bf16_2d(k, "k");
  check_cuda_bf16_2d(v, "v");
  check_cuda_bf16_2d(o, "o");
  TORCH_CHECK(q.size(1) == heads * head_dim, "attention: q width != heads*head_dim");
  TORCH_CHECK(k.size(1) == heads_kv * head_dim && v.size(1) == heads_kv * head_dim, "attention: kv width");
  TORCH_CHECK(o.size(0) == q.size(0) && o.size(1) == q.size(1), "attention: o shape");
  TORCH_CHECK(k.size(0) == v.size(0), "attention: k/v rows");
  if (seg.has_value()) {
    TORCH_CHECK(seg->is_cuda() && seg->scalar_type() == at::kInt && seg->is_contiguous() && seg->numel() == 8 * batch,
                "attention: seg table must be int32 [batch, 8] on the device");
    TORCH_CHECK(max_q_blocks > 0, "attention: max_q_blocks required with a seg table");
  } else if (!cu_q.has_value()) {
    TORCH_CHECK(batch * seq_q == q.size(0) && batch * seq_k == k.size(0), "attention: uniform segment sizes");
  } else {
    TORCH_CHECK(cu_q->scalar_type() == at::kInt && cu_k.has_value() && cu_k->scalar_type() == at::kInt,
                "attention: cu_seqlens must be int32");
    TORCH_CHECK(cu_q->numel() == batch + 1 && cu_k->numel() == batch + 1, "attention: cu_seqlens size");
  }
  if (lse.has_value()) {
    TORCH_CHECK(lse->scalar_type() == at::kFloat && lse->dim() == 2 && lse->size(0) == heads &&
                    lse->size(1) >= q.size(0) && lse->stride(1) == 1,
                "attention: lse must be fp32 [heads, >= tokens]");
  }
  const c10::cuda::CUDAGuard guard(q.device());
  ds::AttnArgs a;
  a.q = q.data_ptr();
  a.q_row_stride = q.stride(0);
  a.k = k.data_ptr();
  a.k_row_stride = k.stride(0);
  a.v = v.data_ptr();
  a.v_row_stride = v.stride(0);
  a.o = o.data_ptr();
  a.o_row_stride = o.stride(0);
  a.lse = lse.has_value() ? lse->data_ptr<float>() : nullptr;
  a.lse_stride = lse.has_value() ? lse->stride(0) : 0;
  a.total_q = static_cast<int>(q.size(0));
  a.total_k = static_cast<int>(k.size(0));
  a.batch = static_cast<int>(batch);
  a.seq_q = static_cast<int>(seq_q);
  a.seq_k = static_cast<int>(seq_k);
  a.cu_seqlens_q = cu_q.has_value() ? cu_q->data_ptr<int>() : nullptr;
  a.cu_seqlens_k = cu_k.has_value() ? cu_k->data_ptr<int>() : nullptr;
  a.max_seq_q = static_cast<int>(max_seq_q);
  a.heads = static_cast<int>(heads);
  a.heads_kv = static_cast<int>(heads_kv);
  a.head_dim = static_cast<int>(head_dim);
  a.softmax_scale = static_cast<float>(scale);
  a.status = status_ptr(status);
  a.seg_table = seg.has_value() ? seg->data_ptr<int>() : nullptr;
  a.max_q_blocks = static_cast<int>(max_q_blocks);
  TORCH_CHECK(k_extra.size() == v_extra.size() && k_extra.size() <= 3, "attention: up to 3 extra KV sources");
  a.kv_sources = 1 + static_cast<int>(k_extra.size());
  for (size_t i = 0; i < k_extra.size(); ++i) {
    check_cuda_bf16_2d(k_extra[i], "k_extra");
    check_cuda_bf16_2d(v_extra[i], "v_extra");
    TORCH_CHECK(k_extra[i].sizes() == k.sizes() && k_extra[i].stride(0) == k.stride(0) &&
                    v_extra[i].sizes() == v.sizes() && v_extra[i].stride(0) == v.stride(0),
                "attention: extra KV sources must match k/v in shape and stride");
    a.k_extra[i] = k_extra[i].data_ptr();
    a.v_extra[i] = v_extra[i].data_ptr();
  }
  TORCH_CHECK(blk_offsets.has_value() == blk_index.has_value(), "attention: give both block-sparse tensors or neither");
  if (blk_offsets.has_value()) {
    // the contents (every block non-empty, tile ids in range) are validated by the caller,
    // which builds the table on the host; here only placement and type
    TORCH_CHECK(blk_offsets->is_cuda() && blk_offsets->scalar_type() == at::kInt && blk_offsets->is_contiguous() &&
                    blk_index->is_cuda() && blk_index->scalar_type() == at::kInt && blk_index->is_contiguous(),
                "attention: block-sparse tables must be contiguous int32 on the device");
    TORCH_CHECK(!seg.has_value() && !cu_q.has_value() && k_extra.empty(),
                "attention: block-sparse needs uniform batches, one KV source and no seg table");
    TORCH_CHECK(blk_offsets->numel() == (seq_q + 255) / 256 + 1, "attention: block-sparse offsets must have one "
                "entry per 256-row query block plus one");
    a.blk_offsets = blk_offsets->data_ptr<int>();
    a.blk_index = blk_index->data_ptr<int>();
  }
  std::vector<at::Tensor> keep;
  if (!seg.has_value() && !cu_q.has_value() && !blk_offsets.has_value() && k_extra.empty() && seq_k > 1024)
    apply_split(a, q.device(), keep);
  ds::launch_attention(a, at::cuda::getCurrentCUDAStream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();  // a failed launch raises here, never passes silently
}

void layernorm_modulate(const at::Tensor& x, at::Tensor& y, const c10::optional<at::Tensor>& scale,
                        const c10::optional<at::Tensor>& shift, int64_t mod_stride, int64_t rows_per_batch,
                        const c10::optional<at::Tensor>& weight, const c10::optional<at::Tensor>& bias,
                        double eps, const c10::optional<at::Tensor>& row_batch) {
  check_cuda_bf16_2d(x, "x");
  check_cuda_bf16_2d(y, "y");
  TORCH_CHECK(x.sizes() == y.sizes(), "layernorm_modulate: shape mismatch");
  if (scale.has_value()) TORCH_CHECK(scale->scalar_type() == at::kFloat, "scale must be fp32");
  if (shift.has_value()) TORCH_CHECK(shift->scalar_type() == at::kFloat, "shift must be fp32");
  if (scale.has_value()) TORCH_CHECK(reinterpret_cast<uintptr_t>(scale->data_ptr()) % 16 == 0, "scale alignment");
  if (shift.has_value()) TORCH_CHECK(reinterpret_cast<uintptr_t>(shift->data_ptr()) % 16 == 0, "shift alignment");
  const c10::cuda::CUDAGuard guard(x.device());
  ds::LayerNormArgs a;
  a.x = x.data_ptr();
  a.x_stride = x.stride(0);
  a.y = y.data_ptr();
  a.y_stride = y.stride(0);
  a.rows = static_cast<int>(x.size(0));
  a.dim = static_cast<int>(x.size(1));
  a.eps = static_cast<float>(eps);
  a.scale = scale.has_value() ? scale->data_ptr<float>() : nullptr;
  a.shift = shift.has_value() ? shift->data_ptr<float>() : nullptr;
  a.mod_stride = mod_stride;
  a.rows_per_batch = static_cast<int>(rows_per_batch);
  a.weight = opt_ptr(weight);
  a.bias = opt_ptr(bias);
  if (row_batch.has_value()) {
    TORCH_CHECK(row_batch->scalar_type() == at::kInt && row_batch->numel() >= x.size(0) && row_batch->is_cuda(),
                "layernorm_modulate: row_batch must be int32 CUDA with one entry per row");
    a.row_batch = row_batch->data_ptr<int>();
  }
  ds::launch_layernorm_modulate(a, at::cuda::getCurrentCUDAStream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();  // a failed launch raises here, never passes silently
}

void rmsnorm_rope(at::Tensor& x, const c10::optional<at::Tensor>& weight, int64_t width, int64_t groups, double eps,
                  const c10::optional<at::Tensor>& cos, const c10::optional<at::Tensor>& sin,
                  int64_t rows_per_batch, int64_t head_dim, const c10::optional<at::Tensor>& weight2,
                  int64_t seg_offset) {
  check_cuda_bf16_2d(x, "x");
  TORCH_CHECK(x.size(1) == width * groups, "rmsnorm_rope: width*groups must equal the view width");
  if (weight2.has_value())
    TORCH_CHECK(seg_offset >= x.size(1) && seg_offset % 8 == 0 && x.stride(0) >= seg_offset + x.size(1),
                "rmsnorm_rope: the second segment must lie beside the first inside the row stride");
  if (cos.has_value()) {
    TORCH_CHECK(sin.has_value() && cos->scalar_type() == at::kFloat && sin->scalar_type() == at::kFloat &&
                    cos->is_contiguous() && sin->is_contiguous(),
                "rmsnorm_rope: cos/sin must be contiguous fp32");
    TORCH_CHECK(cos->size(-1) == head_dim / 2, "rmsnorm_rope: rope table width must be head_dim/2");
    TORCH_CHECK(head_dim % 8 == 0, "rmsnorm_rope: head_dim must be a multiple of 8");
  }
  const c10::cuda::CUDAGuard guard(x.device());
  ds::RmsRopeArgs a;
  a.x = x.data_ptr();
  a.x_stride = x.stride(0);
  a.rows = static_cast<int>(x.size(0));
  a.width = static_cast<int>(width);
  a.groups = static_cast<int>(groups);
  a.weight = opt_ptr(weight);
  a.eps = static_cast<float>(eps);
  a.rope_cos = cos.has_value() ? cos->data_ptr<float>() : nullptr;
  a.rope_sin = sin.has_value() ? sin->data_ptr<float>() : nullptr;
  a.rows_per_batch = static_cast<int>(rows_per_batch);
  a.head_dim = static_cast<int>(head_dim);
  a.weight2 = opt_ptr(weight2);
  a.seg_offset = seg_offset;
  ds::launch_rmsnorm_rope(a, at::cuda::getCurrentCUDAStream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();  // a failed launch raises here, never passes silently
}

const float* opt_f32(const c10::optional<at::Tensor>& t) {
  if (!t.has_value()) return nullptr;
  TORCH_CHECK(t->scalar_type() == at::kFloat && t->is_contiguous(), "sched_step: buffers must be contiguous fp32");
  return t->data_ptr<float>();
}

void sched_step(const at::Tensor& cond, const c10::optional<at::Tensor>& uncond, double guidance, at::Tensor& sample,
                double sigma, bool do_corrector, const c10::optional<at::Tensor>& last, double c_last, double c_x0,
                std::vector<c10::optional<at::Tensor>> c_hist, std::vector<double> c_coef, double p_x, double p_x0,
                double p_v, std::vector<c10::optional<at::Tensor>> p_hist, std::vector<double> p_coef,
                const c10::optional<at::Tensor>& x0_out, const c10::optional<at::Tensor>& last_out) {
  TORCH_CHECK(sample.is_cuda() && sample.scalar_type() == at::kFloat && sample.is_contiguous(),
              "sched_step: sample must be contiguous fp32 CUDA");
  TORCH_CHECK(cond.is_contiguous() && cond.numel() == sample.numel(), "sched_step: cond size");
  TORCH_CHECK(cond.scalar_type() == at::kBFloat16 || cond.scalar_type() == at::kFloat, "sched_step: cond dtype");
  if (uncond.has_value())
    TORCH_CHECK(uncond->is_contiguous() && uncond->scalar_type() == cond.scalar_type() &&
                    uncond->numel() == cond.numel(),
                "sched_step: uncond must match cond");
  TORCH_CHECK(c_hist.size() <= 3 && p_hist.size() <= 3 && c_coef.size() == c_hist.size() &&
                  p_coef.size() == p_hist.size(),
              "sched_step: at most 3 history terms with matching coefficients");
  const c10::cuda::CUDAGuard guard(sample.device());
  ds::SchedStepArgs a;
  a.cond = cond.data_ptr();
  a.uncond = opt_ptr(uncond);
  a.pred_is_bf16 = cond.scalar_type() == at::kBFloat16;
  a.guidance = static_cast<float>(guidance);
  a.n = sample.numel();
  a.sample = sample.data_ptr<float>();
  a.sigma = static_cast<float>(sigma);
  a.do_corrector = do_corrector ? 1 : 0;
  a.last = opt_f32(last);
  TORCH_CHECK(!do_corrector || a.last != nullptr, "sched_step: corrector needs the last sample");
  a.c_last = static_cast<float>(c_last);
  a.c_x0 = static_cast<float>(c_x0);
  for (size_t i = 0; i < c_hist.size(); ++i) {
    a.c_hist_ptr[i] = opt_f32(c_hist[i]);
    a.c_hist[i] = static_cast<float>(c_coef[i]);
  }
  a.p_x = static_cast<float>(p_x);
  a.p_x0 = static_cast<float>(p_x0);
  a.p_v = static_cast<float>(p_v);
  for (size_t i = 0; i < p_hist.size(); ++i) {
    a.p_hist_ptr[i] = opt_f32(p_hist[i]);
    a.p_hist[i] = static_cast<float>(p_coef[i]);
  }
  a.x0_out = x0_out.has_value() ? const_cast<float*>(opt_f32(x0_out)) : nullptr;
  a.last_out = last_out.has_value() ? const_cast<float*>(opt_f32(last_out)) : nullptr;
  ds::launch_sched_step(a, at::cuda::getCurrentCUDAStream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();  // a failed launch raises here, never passes silently
}

// ---------------------------------------------------------------- symmetric heap + fused collectives
std::tuple<at::Tensor, py::bytes> symm_alloc(int64_t nbytes, int64_t device) {
  TORCH_CHECK(nbytes > ds::kFlagBytes, "symmetric heap too small");
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  void* ptr = nullptr;
  C10_CUDA_CHECK(cudaMalloc(&ptr, static_cast<size_t>(nbytes)));
  C10_CUDA_CHECK(cudaMemset(ptr, 0, static_cast<size_t>(nbytes)));
  C10_CUDA_CHECK(cudaDeviceSynchronize());
  cudaIpcMemHandle_t h;
  C10_CUDA_CHECK(cudaIpcGetMemHandle(&h, ptr));
  auto opts = at::TensorOptions().dtype(at::kByte).device(at::kCUDA, device);
  at::Tensor t = torch::from_blob(ptr, {nbytes}, [](void* p) { cudaFree(p); }, opts);
  return {t, py::bytes(reinterpret_cast<const char*>(&h), sizeof(h))};
}

int64_t symm_open(const py::bytes& handle, int64_t device) {
  std::string s = handle;
  TORCH_CHECK(s.size() == sizeof(cudaIpcMemHandle_t), "bad IPC handle");
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  cudaIpcMemHandle_t h;
  std::memcpy(&h, s.data(), sizeof(h));
  void* p = nullptr;
  C10_CUDA_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  return reinterpret_cast<int64_t>(p);
}

void symm_close(int64_t ptr) { cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr)); }

// Lets kernels on `device` read and write `peer`'s memory directly (one process driving
// several GPUs, e.g. the single-process peer-memory probes); true when access is on.
bool peer_enable(int64_t device, int64_t peer) {
  int can = 0;
  C10_CUDA_CHECK(cudaDeviceCanAccessPeer(&can, static_cast<int>(device), static_cast<int>(peer)));
  if (!can) return false;
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  const cudaError_t e = cudaDeviceEnablePeerAccess(static_cast<int>(peer), 0);
  if (e == cudaErrorPeerAccessAlreadyEnabled) {
    (void)cudaGetLastError();
    return true;
  }
  C10_CUDA_CHECK(e);
  return true;
}

ds::PeerGroup make_group(int64_t rank, const std::vector<int64_t>& bases, int64_t timeout_ns) {
  TORCH_CHECK(!bases.empty() && bases.size() <= static_cast<size_t>(ds::kMaxPeers), "group size out of range");
  TORCH_CHECK(rank >= 0 && rank < static_cast<int64_t>(bases.size()), "rank outside the group");
  ds::PeerGroup g;
  g.rank = static_cast<int>(rank);
  g.size = static_cast<int>(bases.size());
  for (size_t i = 0; i < bases.size(); ++i) {
    g.base[i] = reinterpret_cast<void*>(bases[i]);
    g.flags[i] = reinterpret_cast<uint64_t*>(bases[i]);
  }
  g.timeout_ns = static_cast<unsigned long long>(timeout_ns);
  return g;
}

void group_barrier(int64_t rank, const std::vector<int64_t>& bases, int64_t timeout_ns, int64_t channel,
                   int64_t epoch, const at::Tensor& status) {
  ds::launch_group_barrier(make_group(rank, bases, timeout_ns), static_cast<int>(channel),
                           static_cast<uint64_t>(epoch), status_ptr(status), at::cuda::getCurrentCUDAStream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();  // a failed launch raises here, never passes silently
}

void cfg_step_peer(const at::Tensor& mine, int64_t theirs_off, int64_t role, double guidance, at::Tensor& sample,
                   double sigma, bool do_corrector, const c10::optional<at::Tensor>& last, double c_last,
                   double c_x0, std::vector<c10::optional<at::Tensor>> c_hist, std::vector<double> c_coef,
                   double p_x, double p_x0, double p_v, std::vector<c10::optional<at::Tensor>> p_hist,
                   std::vector<double> p_coef, const c10::optional<at::Tensor>& x0_out,
                   const c10::optional<at::Tensor>& last_out, int64_t rank, const std::vector<int64_t>& bases,
                   int64_t timeout_ns, int64_t channel, int64_t epoch, const at::Tensor& status,
                   const c10::optional<at::Tensor>& delta_out) {
  TORCH_CHECK(mine.scalar_type() == at::kBFloat16 && mine.is_contiguous() && mine.numel() == sample.numel(),
              "cfg_step_peer: prediction must be contiguous bf16 of the latent size");
  TORCH_CHECK(sample.scalar_type() == at::kFloat && sample.is_contiguous(), "cfg_step_peer: sample fp32");
  const c10::cuda::CUDAGuard guard(sample.device());
  ds::SchedStepArgs a;
  a.guidance = static_cast<float>(guidance);
  a.n = sample.numel();
  a.sample = sample.data_ptr<float>();
  a.sigma = static_cast<float>(sigma);
  a.do_corrector = do_corrector ? 1 : 0;
  a.last = opt_f32(last);
  a.c_last = static_cast<float>(c_last);
  a.c_x0 = static_cast<float>(c_x0);
  for (size_t i = 0; i < c_hist.size() && i < 3; ++i) {
    a.c_hist_ptr[i] = opt_f32(c_hist[i]);
    a.c_hist[i] = static_cast<float>(c_coef[i]);
  }
  a.p_x = static_cast<float>(p_x);
  a.p_x0 = static_cast<float>(p_x0);
  a.p_v = static_cast<float>(p_v);
  for (size_t i = 0; i < p_hist.size() && i < 3; ++i) {
    a.p_hist_ptr[i] = opt_f32(p_hist[i]);
    a.p_hist[i] = static_cast<float>(p_coef[i]);
  }
  a.x0_out = x0_out.has_value() ? const_cast<float*>(opt_f32(x0_out)) : nullptr;
  a.last_out = last_out.has_value() ? const_cast<float*>(opt_f32(last_out)) : nullptr;
  if (delta_out.has_value()) {
    TORCH_CHECK(delta_out->scalar_type() == at::kFloat && delta_out->is_contiguous() &&
                    delta_out->numel() == sample.numel(),
                "cfg_step_peer: delta_out must be contiguous fp32 of the latent size");
    a.delta_out = delta_out->data_ptr<float>();
  }
  ds::launch_cfg_step_peer(a, make_group(rank, bases, timeout_ns), static_cast<int>(channel),
                           static_cast<uint64_t>(epoch), mine.data_ptr(), theirs_off, static_cast<int>(role),
                           status_ptr(status), at::cuda::getCurrentCUDAStream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();  // a failed launch raises here, never passes silently
}

void qkv_scatter(const at::Tensor& qkv, const at::Tensor& wq, const at::Tensor& wk, double eps,
                 const c10::optional<at::Tensor>& cos, const c10::optional<at::Tensor>& sin, int64_t seq_local,
                 int64_t heads, int64_t head_dim, int64_t rank, const std::vector<int64_t>& bases, int64_t timeout_ns,
                 int64_t recv_off, int64_t pos_base) {
  check_cuda_bf16_2d(qkv, "qkv");
  TORCH_CHECK(qkv.size(1) >= 3 * heads * head_dim, "qkv_scatter: qkv too narrow");
  TORCH_CHECK(qkv.size(0) % seq_local == 0, "qkv_scatter: rows must be batch * seq_local");
  const c10::cuda::CUDAGuard guard(qkv.device());
  ds::QkvScatterArgs a;
  a.qkv = qkv.data_ptr();
  a.qkv_stride = qkv.stride(0);
  a.rows = static_cast<int>(qkv.size(0));
  a.seq_local = static_cast<int>(seq_local);
  a.heads = static_cast<int>(heads);
  a.head_dim = static_cast<int>(head_dim);
  a.wq = wq.data_ptr();
  a.wk = wk.data_ptr();
  a.eps = static_cast<float>(eps);
  a.rope_cos = cos.has_value() ? cos->data_ptr<float>() : nullptr;
  a.rope_sin = sin.has_value() ? sin->data_ptr<float>() : nullptr;
  a.group = make_group(rank, bases, timeout_ns);
  a.recv_off = recv_off;
  a.pos_base = static_cast<int>(pos_base);
  ds::launch_qkv_scatter(a, at::cuda::getCurrentCUDAStream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();  // a failed launch raises here, never passes silently
}

// Dense uniform-batch attention with the timeline of one CTA recorded into `trace`
// (int64 [32 * 24], SM clock stamps); profiling only.
void attention_trace(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, at::Tensor& o, int64_t batch,
                     int64_t seq, int64_t heads, int64_t head_dim, double scale, const at::Tensor& status,
                     at::Tensor& trace) {
  check_cuda_bf16_2d(q, "q");
  check_cuda_bf16_2d(k, "k");
  check_cuda_bf16_2d(v, "v");
  check_cuda_bf16_2d(o, "o");
  TORCH_CHECK(q.size(0) == batch * seq && k.size(0) == batch * seq && v.size(0) == batch * seq &&
                  q.size(1) == heads * head_dim && o.sizes() == q.sizes(),
              "attention_trace: shapes");
  TORCH_CHECK(trace.is_cuda() && trace.scalar_type() == at::kLong && trace.is_contiguous() && trace.numel() >= 32 * 24,
              "attention_trace: trace must be int64 [>= 768] on the device");
  const c10::cuda::CUDAGuard guard(q.device());
  ds::AttnArgs a;
  a.q = q.data_ptr();
  a.q_row_stride = q.stride(0);
  a.k = k.data_ptr();
  a.k_row_stride = k.stride(0);
  a.v = v.data_ptr();
  a.v_row_stride = v.stride(0);
  a.o = o.data_ptr();
  a.o_row_stride = o.stride(0);
  a.total_q = a.total_k = static_cast<int>(q.size(0));
  a.batch = static_cast<int>(batch);
  a.seq_q = a.seq_k = static_cast<int>(seq);
  a.heads = a.heads_kv = static_cast<int>(heads);
  a.head_dim = static_cast<int>(head_dim);
  a.softmax_scale = static_cast<float>(scale);
  a.status = status_ptr(status);
  a.trace = reinterpret_cast<unsigned long long*>(trace.data_ptr<int64_t>());
  ds::launch_attention(a, at::cuda::getCurrentCUDAStream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void attention_scatter(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, int64_t batch, int64_t seq,
                       int64_t heads, int64_t head_dim, double scale, int64_t rank, const std::vector<int64_t>& bases,
                       int64_t timeout_ns, int64_t o_off, int64_t seq_local, int64_t head_offset,
                       int64_t peer_stride, const at::Tensor& status, std::vector<int64_t> k_extra_ptrs,
                       std::vector<int64_t> v_extra_ptrs) {
  check_cuda_bf16_2d(q, "q");
  check_cuda_bf16_2d(k, "k");
  check_cuda_bf16_2d(v, "v");
  TORCH_CHECK(q.size(0) == batch * seq && k.size(0) == batch * seq, "attention_scatter: rows");
  const c10::cuda::CUDAGuard guard(q.device());
  ds::AttnArgs a;
  a.q = q.data_ptr();
  a.q_row_stride = q.stride(0);
  a.k = k.data_ptr();
  a.k_row_stride = k.stride(0);
  a.v = v.data_ptr();
  a.v_row_stride = v.stride(0);
  a.o = nullptr;
  a.total_q = static_cast<int>(q.size(0));
  a.total_k = static_cast<int>(k.size(0));
  a.batch = static_cast<int>(batch);
  a.seq_q = a.seq_k = static_cast<int>(seq);
  a.heads = a.heads_kv = static_cast<int>(heads);
  a.head_dim = static_cast<int>(head_dim);
  a.softmax_scale = static_cast<float>(scale);
  a.status = status_ptr(status);
  a.o_scatter = 1;
  a.o_group = make_group(rank, bases, timeout_ns);
  a.o_off = o_off;
  a.o_seq_local = static_cast<int>(seq_local);
  a.o_head_offset = static_cast<int>(head_offset);
  a.o_peer_stride = peer_stride;
  TORCH_CHECK(k_extra_ptrs.size() == v_extra_ptrs.size() && k_extra_ptrs.size() <= 3, "up to 3 ring peers");
  a.kv_sources = 1 + static_cast<int>(k_extra_ptrs.size());
  for (size_t i = 0; i < k_extra_ptrs.size(); ++i) {
    a.k_extra[i] = reinterpret_cast<const void*>(k_extra_ptrs[i]);
    a.v_extra[i] = reinterpret_cast<const void*>(v_extra_ptrs[i]);
  }
  std::vector<at::Tensor> keep;
  if (k_extra_ptrs.empty() && seq > 1024) apply_split(a, q.device(), keep);
  ds::launch_attention(a, at::cuda::getCurrentCUDAStream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();  // a failed launch raises here, never passes silently
}

void allgather_rows(const at::Tensor& src, int64_t dst_off, int64_t rank, const std::vector<int64_t>& bases,
                    int64_t timeout_ns) {
  TORCH_CHECK(src.is_cuda() && src.is_contiguous(), "allgather_rows: contiguous CUDA source");
  const c10::cuda::CUDAGuard guard(src.device());
  ds::launch_allgather_rows(make_group(rank, bases, timeout_ns), src.data_ptr(),
                            static_cast<int64_t>(src.numel() * src.element_size()), dst_off,
                            at::cuda::getCurrentCUDAStream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();  // a failed launch raises here, never passes silently
}

void strided_put(const at::Tensor& src, int64_t peer, int64_t dst_off, int64_t rank,
                 const std::vector<int64_t>& bases, int64_t timeout_ns) {
  TORCH_CHECK(src.is_cuda() && src.dim() <= 4, "strided_put: CUDA tensor of at most 4 dims");
  TORCH_CHECK(src.element_size() == 2 || src.element_size() == 4, "strided_put: 2- or 4-byte elements");
  const c10::cuda::CUDAGuard guard(src.device());
  ds::StridedSlice sl;
  sl.esize = static_cast<int>(src.element_size());
  const int off = 4 - static_cast<int>(src.dim());
  for (int d = 0; d < src.dim(); ++d) {
    sl.size[off + d] = src.size(d);
    sl.stride[off + d] = src.stride(d) * src.element_size();
  }
  ds::launch_strided_put(make_group(rank, bases, timeout_ns), static_cast<int>(peer), src.data_ptr(), sl, dst_off,
                         at::cuda::getCurrentCUDAStream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();  // a failed launch raises here, never passes silently
}

void group_flag(int64_t rank, const std::vector<int64_t>& bases, int64_t timeout_ns, int64_t channel, int64_t epoch,
                int64_t flag, const at::Tensor& out, const at::Tensor& status) {
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kInt && out.numel() >= 1, "group_flag: int32 CUDA output");
  const c10::cuda::CUDAGuard guard(out.device());
  ds::launch_group_flag(make_group(rank, bases, timeout_ns), static_cast<int>(channel), static_cast<uint64_t>(epoch),
                        static_cast<int>(flag), out.data_ptr<int>(), status_ptr(status),
                        at::cuda::getCurrentCUDAStream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();  // a failed launch raises here, never passes silently
}

void conv(const at::Tensor& x, const at::Tensor& w, at::Tensor& y, const c10::optional<at::Tensor>& bias,
          const c10::optional<at::Tensor>& residual, int64_t kt, int64_t kh, int64_t kw, int64_t pad_h, int64_t pad_w,
          const at::Tensor& status, int64_t bn_override) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 4 && x.is_contiguous(),
              "conv: x must be contiguous bf16 [T, H, W, C]");
  TORCH_CHECK(y.is_cuda() && y.scalar_type() == at::kBFloat16 && y.dim() == 4 && y.is_contiguous(),
              "conv: y must be contiguous bf16 [T, H, W, C_out]");
  TORCH_CHECK(w.is_cuda() && w.scalar_type() == at::kBFloat16 && w.dim() == 2 && w.is_contiguous(),
              "conv: w must be contiguous bf16 [C_out_pad, KT*KH*KW*C_in]");
  TORCH_CHECK(w.size(1) == kt * kh * kw * x.size(3), "conv: weight K does not match the kernel and C_in");
  TORCH_CHECK(y.size(0) == x.size(0) - kt + 1 && y.size(1) == x.size(1) + 2 * pad_h - kh + 1 &&
                  y.size(2) == x.size(2) + 2 * pad_w - kw + 1 && y.size(3) <= w.size(0),
              "conv: output shape mismatch");
  if (bias.has_value())
    TORCH_CHECK(bias->is_contiguous() && bias->scalar_type() == at::kBFloat16 && bias->numel() == w.size(0),
                "conv: bias must be contiguous bf16 [C_out_pad]");
  if (residual.has_value())
    TORCH_CHECK(residual->is_contiguous() && residual->scalar_type() == at::kBFloat16 && residual->sizes() == y.sizes(),
                "conv: residual must be contiguous bf16 shaped like y");
  const c10::cuda::CUDAGuard guard(x.device());
  ds::ConvArgs a;
  a.X = x.data_ptr();
  a.W = w.data_ptr();
  a.Y = y.data_ptr();
  a.bias = opt_ptr(bias);
  a.R = opt_ptr(residual);
  a.T_in = static_cast<int>(x.size(0));
  a.H_in = static_cast<int>(x.size(1));
  a.W_in = static_cast<int>(x.size(2));
  a.C_in = static_cast<int>(x.size(3));
  a.C_out = static_cast<int>(y.size(3));
  a.C_out_pad = static_cast<int>(w.size(0));
  a.KT = static_cast<int>(kt);
  a.KH = static_cast<int>(kh);
  a.KW = static_cast<int>(kw);
  a.pad_h = static_cast<int>(pad_h);
  a.pad_w = static_cast<int>(pad_w);
  a.status = status_ptr(status);
  a.bn_override = static_cast<int>(bn_override);
  ds::launch_conv(a, at::cuda::getCurrentCUDAStream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();  // a failed launch raises here, never passes silently
}

ds::RingCodecArgs ring_args(int64_t rows, int64_t heads, int64_t head_dim, int64_t src, int64_t slot_off,
                           int64_t slot_bytes, int64_t rank, const std::vector<int64_t>& bases, int64_t timeout_ns) {
  ds::RingCodecArgs a;
  a.rows = static_cast<int>(rows);
  a.heads = static_cast<int>(heads);
  a.head_dim = static_cast<int>(head_dim);
  a.src = static_cast<int>(src);
  a.slot_off = slot_off;
  a.slot_bytes = slot_bytes;
  a.group = make_group(rank, bases, timeout_ns);
  return a;
}

void ring_quant_push(const at::Tensor& kv, int64_t heads, int64_t head_dim, int64_t src, int64_t slot_off,
                     int64_t slot_bytes, int64_t rank, const std::vector<int64_t>& bases, int64_t timeout_ns) {
  check_cuda_bf16_2d(kv, "kv");
  TORCH_CHECK(kv.size(1) >= 2 * heads * head_dim, "ring_quant_push: kv narrower than K and V");
  const c10::cuda::CUDAGuard guard(kv.device());
  ds::RingCodecArgs a = ring_args(kv.size(0), heads, head_dim, src, slot_off, slot_bytes, rank, bases, timeout_ns);
  a.kv = kv.data_ptr();
  a.kv_stride = kv.stride(0);
  ds::launch_ring_quant_push(a, at::cuda::getCurrentCUDAStream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();  // a failed launch raises here, never passes silently
}

void ring_dequant(at::Tensor& out, int64_t heads, int64_t head_dim, int64_t src, int64_t slot_off, int64_t slot_bytes,
                  int64_t rank, const std::vector<int64_t>& bases, int64_t timeout_ns) {
  check_cuda_bf16_2d(out, "out");
  TORCH_CHECK(out.size(1) >= 3 * heads * head_dim, "ring_dequant: out must be [rows, >= 3*heads*head_dim]");
  const c10::cuda::CUDAGuard guard(out.device());
  ds::RingCodecArgs a = ring_args(out.size(0), heads, head_dim, src, slot_off, slot_bytes, rank, bases, timeout_ns);
  ds::launch_ring_dequant(a, static_cast<int>(src), out.data_ptr(), out.stride(0), at::cuda::getCurrentCUDAStream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();  // a failed launch raises here, never passes silently
}

void put_peers(const at::Tensor& src, int64_t mask, int64_t dst_off, int64_t rank, const std::vector<int64_t>& bases,
               int64_t timeout_ns) {
  TORCH_CHECK(src.is_cuda() && src.is_contiguous(), "put_peers: contiguous CUDA source");
  const c10::cuda::CUDAGuard guard(src.device());
  ds::launch_put_peers(make_group(rank, bases, timeout_ns), static_cast<unsigned>(mask), src.data_ptr(),
                       static_cast<int64_t>(src.numel() * src.element_size()), dst_off,
                       at::cuda::getCurrentCUDAStream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();  // a failed launch raises here, never passes silently
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "sm_100a kernels of ditserve_b200 (tcgen05 GEMM/attention, fused norms, solver step)";
  m.def("gemm", &gemm, "C = epilogue(A @ B^T)");
  m.def("gemm_pick_bn", &ds::gemm_pick_bn);
  m.def("attention", &attention, "non-causal flash attention (tcgen05/TMEM)");
  m.def("layernorm_modulate", &layernorm_modulate, "LayerNorm + adaLN modulation");
  m.def("rmsnorm_rope", &rmsnorm_rope, "RMS norm + interleaved RoPE, in place");
  m.def("sched_step", &sched_step, "CFG combine + UniPC/Euler latent update");
  m.def("symm_alloc", &symm_alloc, "allocate a zeroed symmetric heap and its IPC handle");
  m.def("symm_open", &symm_open, "open a peer heap from its IPC handle");
  m.def("symm_close", &symm_close);
  m.def("peer_enable", &peer_enable, "enable direct access from one device to a peer's memory (same process)");
  m.def("group_barrier", &group_barrier, "bounded flag barrier over peer memory");
  m.def("cfg_step_peer", &cfg_step_peer, "CFG exchange over NVLink fused with guidance + latent update");
  m.def("qkv_scatter", &qkv_scatter, "RMS qk-norm + RoPE + Ulysses all-to-all scatter");
  m.def("attention_tail_split_parts", [](int64_t batch, int64_t seq_q, int64_t seq_k, int64_t heads, int64_t sms) {
    return tail_split_parts(((seq_q + 255) / 256) * heads * batch, (seq_k + 127) / 128, sms);
  }, "key ranges the attention grid gives its tail units (1: no split) for a shape on `sms` SMs");
  m.def("attention_trace", &attention_trace, "attention with a one-CTA clock timeline (profiling)");
  m.def("attention_scatter", &attention_scatter, "attention with the head->sequence all-to-all in its epilogue");
  m.def("allgather_rows", &allgather_rows, "sequence all-gather by peer stores");
  m.def("strided_put", &strided_put, "strided slice -> contiguous buffer of a group member (halo exchange)");
  m.def("group_flag", &group_flag, "doorbell flag MAX over a peer group (one launch, bounded waits)");
  m.def("put_peers", &put_peers, "copy a buffer into several group members' heaps");
  m.def("conv", &conv, "implicit-GEMM convolution, channels-last (tcgen05/TMEM)");
  m.def("ring_quant_push", &ring_quant_push, "INT8-quantize this rank's ring K/V chunk into every ring peer's slot");
  m.def("ring_dequant", &ring_dequant, "dequantize one peer's INT8 ring slot into a local bf16 [rows, 3w] buffer");
  m.def("ring_slot_bytes", &ds::ring_slot_bytes, "bytes of one INT8 ring slot");
  m.attr("FLAG_BYTES") = ds::kFlagBytes;
  m.attr("MAX_PEERS") = ds::kMaxPeers;
  m.attr("CHANNELS") = ds::kChannels;
}
