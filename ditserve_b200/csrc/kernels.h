// C++ launch interface of the sm_100a kernels.  Plain structs of raw device
// pointers so the .cu files never include torch headers (fast builds); the
// torch bindings in bindings.cpp fill these from tensors.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>
#include <stdexcept>

namespace ds {

enum GemmEpilogue : int { kEpiNone = 0, kEpiGelu = 1, kEpiGatedRes = 2, kEpiRes = 3 };

struct GemmArgs {
  const void* A = nullptr;  // [M, K] bf16, row stride lda
  int64_t lda = 0;
  const void* B = nullptr;  // [N, K] bf16, row stride ldb
  int64_t ldb = 0;
  void* C = nullptr;  // [M, N] bf16, row stride ldc
  int64_t ldc = 0;
  int M = 0, N = 0, K = 0;
  const void* bias = nullptr;  // [N] bf16 or null
  int epilogue = kEpiNone;
  const void* R = nullptr;  // residual [M, N] bf16, row stride ldr (may alias C)
  int64_t ldr = 0;
  const float* gate = nullptr;  // gate[b * gate_stride + n], b = row / rows_per_batch
  int64_t gate_stride = 0;
  int rows_per_batch = 0;
  int* status = nullptr;  // device status word pair (code, site)
  int num_sms = 0;        // 0: all SMs of the current device
  int bn_override = 0;    // 0: heuristic
};
void launch_gemm(const GemmArgs& a, cudaStream_t stream);
int gemm_pick_bn(int M, int N);

// Flash attention (non-causal) over bf16 [tokens, heads*D] row-major views.
// Segments: either uniform (batch x seq_q / seq_k) or ragged through
// cu_seqlens_q / cu_seqlens_k (int32, batch+1 entries, device memory).
struct AttnArgs {
  const void* q = nullptr;
  int64_t q_row_stride = 0;  // elements between consecutive tokens
  const void* k = nullptr;
  int64_t k_row_stride = 0;
  const void* v = nullptr;
  int64_t v_row_stride = 0;
  void* o = nullptr;
  int64_t o_row_stride = 0;
  float* lse = nullptr;  // optional [heads, total_q] natural-log LSE (fp32)
  int64_t lse_stride = 0;
  int total_q = 0, total_k = 0;  // rows of the q/k tensors (TMA bounds)
  int batch = 1;
  int seq_q = 0, seq_k = 0;  // uniform lengths when cu_seqlens are null
  const int* cu_seqlens_q = nullptr;
  const int* cu_seqlens_k = nullptr;
  int max_seq_q = 0;
  int heads = 0, heads_kv = 0, head_dim = 128;
  float softmax_scale = 0.f;
  int* status = nullptr;
};
void launch_attention(const AttnArgs& a, cudaStream_t stream);

// LayerNorm (no affine, or affine w/b) followed by adaLN modulation:
//   y = LN(x) * (1 + scale[b]) + shift[b]       (scale/shift fp32 rows)
//   y = LN(x) * w + b                           (affine, when w != null)
struct LayerNormArgs {
  const void* x = nullptr;
  int64_t x_stride = 0;
  void* y = nullptr;
  int64_t y_stride = 0;
  int rows = 0, dim = 0;
  float eps = 1e-6f;
  const float* scale = nullptr;  // [B, dim] with stride mod_stride
  const float* shift = nullptr;
  int64_t mod_stride = 0;
  int rows_per_batch = 0;
  const void* weight = nullptr;  // bf16 [dim]
  const void* bias = nullptr;    // bf16 [dim]
};
void launch_layernorm_modulate(const LayerNormArgs& a, cudaStream_t stream);

// RMS norm (optionally across all heads of a row, or per head) with an
// optional rotary embedding on interleaved pairs, in place on a bf16 view.
struct RmsRopeArgs {
  void* x = nullptr;
  int64_t x_stride = 0;  // elements between tokens
  int rows = 0;
  int width = 0;          // elements normalised per row-group (H*D or D)
  int groups = 1;         // groups per row (1: norm across heads; H: per head)
  const void* weight = nullptr;  // bf16 [width]
  float eps = 1e-6f;
  const float* rope_cos = nullptr;  // [rows_per_batch, head_dim/2] fp32 or null
  const float* rope_sin = nullptr;
  int rows_per_batch = 0;
  int head_dim = 128;
};
void launch_rmsnorm_rope(const RmsRopeArgs& a, cudaStream_t stream);

// CFG combine + scheduler update in one pass over an fp32 latent.
//   v  = uncond + g * (cond - uncond)          (v = cond when uncond is null)
//   x0 = x - sigma * v                          (flow prediction -> data)
//   xc = do_corrector ? c_last*last + c_x0*x0 + sum_j c_hist[j]*hist[j] : x
//   x' = p_x*xc + p_x0*x0 + p_v*v + sum_j p_hist[j]*hist[j]
// Every coefficient comes from the host-side scheduler (UniPC bh2 predictor /
// corrector, or flow-matching Euler with p_x = 1, p_v = dt).  Optional outputs
// store x0 (history for the next step) and xc (the corrected sample that the
// next corrector starts from).  Outputs may alias inputs element-wise.
struct SchedStepArgs {
  const void* cond = nullptr;
  const void* uncond = nullptr;
  int pred_is_bf16 = 1;
  float guidance = 1.f;
  int64_t n = 0;
  float* sample = nullptr;  // in: x, out: x'
  float sigma = 0.f;
  int do_corrector = 0;
  const float* last = nullptr;
  float c_last = 0.f, c_x0 = 0.f;
  const float* c_hist_ptr[3] = {nullptr, nullptr, nullptr};
  float c_hist[3] = {0.f, 0.f, 0.f};
  float p_x = 1.f, p_x0 = 0.f, p_v = 0.f;
  const float* p_hist_ptr[3] = {nullptr, nullptr, nullptr};
  float p_hist[3] = {0.f, 0.f, 0.f};
  float* x0_out = nullptr;
  float* last_out = nullptr;
};
void launch_sched_step(const SchedStepArgs& a, cudaStream_t stream);

}  // namespace ds
