// C++ launch interface of the sm_100a kernels.  Plain structs of raw device
// pointers so the .cu files never include torch headers (fast builds); the
// torch bindings in bindings.cpp fill these from tensors.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>
#include <stdexcept>

namespace ds {

constexpr int kMaxPeers = 8;
constexpr int kChannels = 16;
// Flag area at the head of every symmetric heap: uint64 flags[kChannels][kMaxPeers].
constexpr int64_t kFlagBytes = static_cast<int64_t>(kChannels) * kMaxPeers * 8;

// A rank group over symmetric heaps: base[i] is member i's heap (peer-mapped),
// flags[i] its flag area (= base[i]).  rank/size are positions inside the group.
struct PeerGroup {
  int rank = 0, size = 1;
  void* base[kMaxPeers] = {};
  uint64_t* flags[kMaxPeers] = {};
  unsigned long long timeout_ns = 10000000000ull;
};

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
  const int* row_batch = nullptr;  // optional per-row batch index (packed ragged batches)
  int* status = nullptr;  // device status word pair (code, site)
  int num_sms = 0;        // 0: all SMs of the current device
  int bn_override = 0;    // 0: heuristic
  int cta_pair = -1;      // CTA-pair (cta_group::2) kernel: 1 on, 0 off, -1 default (DS_GEMM_PAIR, else on)
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
  // extra key/value sources with the same shape and strides as k/v (ring attention: the
  // chunks of the ring peers, read in place); every segment attends to all sources
  int kv_sources = 1;
  const void* k_extra[3] = {nullptr, nullptr, nullptr};
  const void* v_extra[3] = {nullptr, nullptr, nullptr};
  const int* seg_table = nullptr;  // [batch][8]: qa0 qa1 qb0 qb1 ka0 ka1 kb0 kb1 (dual-range segments)
  int max_q_blocks = 0;            // grid.x in dual-range mode: max over segments of 256-row query blocks
  int heads = 0, heads_kv = 0, head_dim = 128;
  float softmax_scale = 0.f;
  int* status = nullptr;
  // peer-store epilogue (Ulysses head->sequence all-to-all): when o_scatter is set, the
  // output row of query token t (of S = size*o_seq_local) is stored on group member
  // t / o_seq_local at heap offset o_off, row (b*o_seq_local + t % o_seq_local), column
  // (o_head_offset + h) * head_dim, row stride o_peer_stride elements.
  int o_scatter = 0;
  PeerGroup o_group;
  int64_t o_off = 0;
  int o_seq_local = 0;
  int o_head_offset = 0;
  int64_t o_peer_stride = 0;
  // block-sparse attention: int32 CSR over query blocks of 256 rows (grid.x); query block qb
  // attends only to the 128-key tiles blk_index[blk_offsets[qb] .. blk_offsets[qb + 1]) of its
  // segment, every block naming at least one tile (one KV source, no dual-range table)
  const int* blk_offsets = nullptr;
  const int* blk_index = nullptr;
  // optional timeline of one CTA (SM clock stamps, [32 tiles][24 events]); profiling only
  unsigned long long* trace = nullptr;
  // optional work list (uniform batches, one KV source): CTA i runs work[i] =
  // {query block | (partial slot + 1) << 16, head, batch, first key tile | end tile << 16};
  // partial slots leave fp32 O [slots][256][head_dim] in part_o and (max, sum) [slots][256]
  // in part_ml, and merge_units[u] = {query block, head, batch, first slot | parts << 16}
  // name the units whose parts attention_merge combines into the output
  const int4* work = nullptr;
  int num_work = 0;
  float* part_o = nullptr;
  float* part_ml = nullptr;
  const int4* merge_units = nullptr;
  int num_merge_units = 0;
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
  const int* row_batch = nullptr;  // optional per-row batch index (packed ragged batches)
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
  const void* weight2 = nullptr;  // second segment (e.g. k beside q): its weight, or null for one segment
  int64_t seg_offset = 0;         // elements from the first segment to the second within a row
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
  float* delta_out = nullptr;  // optional: cond - uncond (fp32), for late-step CFG folding
};
void launch_sched_step(const SchedStepArgs& a, cudaStream_t stream);

// ---- fused collectives over peer memory (comm.cu) ----
struct QkvScatterArgs {
  const void* qkv = nullptr;  // [rows = B*Sl, >= 3*H*D] bf16
  int64_t qkv_stride = 0;
  int rows = 0, seq_local = 0, heads = 0, head_dim = 128;
  const void* wq = nullptr;  // bf16 [H*D] RMS weights
  const void* wk = nullptr;
  float eps = 1e-6f;
  const float* rope_cos = nullptr;  // [S_full, D/2] (global positions)
  const float* rope_sin = nullptr;
  PeerGroup group;
  int64_t recv_off = 0;  // heap offset of every member's receive buffer [B*S, 3*Hl*D]
  int pos_base = 0;      // global position of this group's first token (ring chunk offset)
};
void launch_group_barrier(const PeerGroup& g, int channel, uint64_t epoch, int* status, cudaStream_t s);
void launch_cfg_step_peer(const SchedStepArgs& a, const PeerGroup& g, int channel, uint64_t epoch,
                          const void* mine, int64_t theirs_off, int my_role, int* status, cudaStream_t s);
void launch_qkv_scatter(const QkvScatterArgs& a, cudaStream_t s);
void launch_allgather_rows(const PeerGroup& g, const void* src, int64_t bytes, int64_t dst_off, cudaStream_t s);
struct StridedSlice {
  int64_t size[4] = {1, 1, 1, 1};
  int64_t stride[4] = {0, 0, 0, 0};  // bytes
  int esize = 2;
};
void launch_strided_put(const PeerGroup& g, int peer, const void* src, const StridedSlice& sl, int64_t dst_off,
                        cudaStream_t s);
// MAX of a 0/1 flag over the group (out: 0/1, or -1 after a peer timeout).
// ---- implicit-GEMM convolution, channels-last (conv.cu) ----
struct ConvArgs {
  const void* X = nullptr;   // [T_in, H_in, W_in, C_in] bf16
  const void* W = nullptr;   // [C_out_pad, KT*KH*KW*C_in] bf16 (tap-major, then C_in)
  void* Y = nullptr;         // [T_out, H_out, W_out, C_out] bf16
  const void* bias = nullptr;  // bf16 [C_out_pad] or null
  const void* R = nullptr;     // residual, Y's layout, or null
  int T_in = 0, H_in = 0, W_in = 0, C_in = 0, C_out = 0, C_out_pad = 0;
  int KT = 1, KH = 3, KW = 3, pad_h = 1, pad_w = 1;
  int* status = nullptr;
  int bn_override = 0;
};
int conv_pick_bn(int c_out_pad);
void launch_conv(const ConvArgs& a, cudaStream_t stream);

// ---- INT8 ring K/V transport (ring_codec.cu) ----
struct RingCodecArgs {
  const void* kv = nullptr;  // bf16 rows: K at column 0, V at column heads*head_dim (row stride kv_stride)
  int64_t kv_stride = 0;
  int rows = 0, heads = 0, head_dim = 128;
  int src = 0;               // slot index of this rank's packet (its position in the ring group)
  int64_t slot_off = 0;      // heap offset of slot 0 in every member
  int64_t slot_bytes = 0;    // >= ring_slot_bytes(rows, heads, head_dim)
  PeerGroup group;           // the ring group
};
int64_t ring_slot_bytes(int rows, int heads, int head_dim);
void launch_ring_quant_push(const RingCodecArgs& a, cudaStream_t s);
void launch_ring_dequant(const RingCodecArgs& a, int src, void* out, int64_t out_stride, cudaStream_t s);
void launch_group_flag(const PeerGroup& g, int channel, uint64_t epoch, int flag, int* out, int* status,
                       cudaStream_t s);
// Copy `bytes` (16-byte multiple) from src to offset dst_off of every member in `mask`.
void launch_put_peers(const PeerGroup& g, unsigned mask, const void* src, int64_t bytes, int64_t dst_off,
                      cudaStream_t s);

}  // namespace ds
