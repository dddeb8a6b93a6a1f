// Memory-bound fused kernels of the DiT block and the solver step (sm_100a).
//
//  * layernorm_modulate: fp32 LayerNorm of a bf16 row followed by the adaLN
//    modulation  y = LN(x) * (1 + scale[b]) + shift[b]  (or an affine LN).
//    Replaces `norm1(h.float()) * (1 + scale) + shift` of the reference's Wan
//    block (workers/ditserve/models/wan/block.py:282-297) and the packed
//    adaLN-Zero of SD3.5 (workers/ditserve/models/sd35_batch.py:336-394).
//  * rmsnorm_rope: RMS norm across all heads (Wan qk-norm) or per head
//    (SD3.5 qk-norm), then the interleaved-pair rotary embedding, in place on
//    the q or k columns of the fused QKV projection output
//    (workers/xfuser/model_executor/models/transformers/transformer_wan.py:158-191).
//  * sched_step: classifier-free-guidance combine fused with the UniPC /
//    flow-matching Euler latent update (workers/ditserve/models/wan/block.py:472-486,
//    workers/ditserve/models/sd35.py:943-952).
// One warp owns one row; every global access is a 16-byte vector.
#include "sm100.cuh"
#include "kernels.h"

namespace ds {
namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&f)[8]) {
  uint4 u = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = unpack_bf16x2(w[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ void store8(__nv_bfloat16* p, const float (&f)[8]) {
  uint4 u;
  u.x = pack_bf16x2(f[0], f[1]);
  u.y = pack_bf16x2(f[2], f[3]);
  u.z = pack_bf16x2(f[4], f[5]);
  u.w = pack_bf16x2(f[6], f[7]);
  *reinterpret_cast<uint4*>(p) = u;
}

// kChunks = dim / 256 (8 bf16 per lane per chunk); rows stay in registers.
template <int kChunks>
__global__ void __launch_bounds__(256) layernorm_modulate_kernel(LayerNormArgs a) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= a.rows) return;
  const __nv_bfloat16* x = reinterpret_cast<const __nv_bfloat16*>(a.x) + static_cast<int64_t>(warp) * a.x_stride;
  __nv_bfloat16* y = reinterpret_cast<__nv_bfloat16*>(a.y) + static_cast<int64_t>(warp) * a.y_stride;
  float v[kChunks][8];
  float s = 0.f;
#pragma unroll
  for (int c = 0; c < kChunks; ++c) {
    load8(x + c * 256 + lane * 8, v[c]);
#pragma unroll
    for (int i = 0; i < 8; ++i) s += v[c][i];
  }
  const float inv_dim = 1.0f / static_cast<float>(a.dim);
  const float mean = warp_sum(s) * inv_dim;
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < kChunks; ++c)
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float d = v[c][i] - mean;
      ss += d * d;
    }
  const float rstd = rsqrtf(warp_sum(ss) * inv_dim + a.eps);
  const int b = a.row_batch != nullptr ? a.row_batch[warp] : (a.rows_per_batch > 0 ? warp / a.rows_per_batch : 0);
  const float* scale = a.scale ? a.scale + static_cast<int64_t>(b) * a.mod_stride : nullptr;
  const float* shift = a.shift ? a.shift + static_cast<int64_t>(b) * a.mod_stride : nullptr;
#pragma unroll
  for (int c = 0; c < kChunks; ++c) {
    const int col = c * 256 + lane * 8;
    float o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = (v[c][i] - mean) * rstd;
    if (a.weight != nullptr) {
      float w[8];
      load8(reinterpret_cast<const __nv_bfloat16*>(a.weight) + col, w);
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] *= w[i];
    }
    if (a.bias != nullptr) {
      float bb[8];
      load8(reinterpret_cast<const __nv_bfloat16*>(a.bias) + col, bb);
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] += bb[i];
    }
    if (scale != nullptr) {
      const float4 s0 = *reinterpret_cast<const float4*>(scale + col);
      const float4 s1 = *reinterpret_cast<const float4*>(scale + col + 4);
      const float sc[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] *= 1.0f + sc[i];
    }
    if (shift != nullptr) {
      const float4 t0 = *reinterpret_cast<const float4*>(shift + col);
      const float4 t1 = *reinterpret_cast<const float4*>(shift + col + 4);
      const float sh[8] = {t0.x, t0.y, t0.z, t0.w, t1.x, t1.y, t1.z, t1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] += sh[i];
    }
    store8(y + col, o);
  }
}

// One warp per row.  kChunks = row width / 256.  kGroupLanes lanes share one
// normalisation group per chunk (32: whole row, 16: 128-wide heads, 8: 64-wide).
// With a second segment (weight2 set) consecutive warps take the two segments of one row (q
// and k of one token, seg_offset elements apart), so one launch normalises both.
template <int kChunks, int kGroupLanes>
__global__ void __launch_bounds__(256) rmsnorm_rope_kernel(RmsRopeArgs a) {
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const bool two = a.weight2 != nullptr;
  const int seg = two ? (gw & 1) : 0;
  const int warp = two ? (gw >> 1) : gw;  // row
  if (warp >= a.rows) return;
  __nv_bfloat16* x = reinterpret_cast<__nv_bfloat16*>(a.x) + static_cast<int64_t>(warp) * a.x_stride +
                     static_cast<int64_t>(seg) * a.seg_offset;
  const void* weight = seg ? a.weight2 : a.weight;
  float v[kChunks][8];
  float part[kChunks];
  float total = 0.f;
#pragma unroll
  for (int c = 0; c < kChunks; ++c) {
    load8(x + c * 256 + lane * 8, v[c]);
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) s += v[c][i] * v[c][i];
    part[c] = s;
    total += s;
  }
  float rinv[kChunks];
  if (kGroupLanes == 32) {
    const float r = rsqrtf(warp_sum(total) / static_cast<float>(a.width) + a.eps);
#pragma unroll
    for (int c = 0; c < kChunks; ++c) rinv[c] = r;
  } else {
#pragma unroll
    for (int c = 0; c < kChunks; ++c) {
      float s = part[c];
#pragma unroll
      for (int o = kGroupLanes / 2; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      rinv[c] = rsqrtf(s / static_cast<float>(a.width) + a.eps);
    }
  }
  const int pos = a.rows_per_batch > 0 ? warp % a.rows_per_batch : warp;
  const int half = a.head_dim / 2;
#pragma unroll
  for (int c = 0; c < kChunks; ++c) {
    const int col = c * 256 + lane * 8;
    const int wcol = kGroupLanes == 32 ? col : (col % a.width);
    float w[8];
    if (weight != nullptr) {
      load8(reinterpret_cast<const __nv_bfloat16*>(weight) + wcol, w);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) w[i] = 1.f;
    }
    float o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = v[c][i] * rinv[c] * w[i];
    if (a.rope_cos != nullptr) {
      // the reference rounds the normalised q/k to the model dtype before RoPE
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = __bfloat162float(__float2bfloat16_rn(o[i]));
      const int pair0 = (col % a.head_dim) / 2;
      const float4 c4 = *reinterpret_cast<const float4*>(a.rope_cos + static_cast<int64_t>(pos) * half + pair0);
      const float4 s4 = *reinterpret_cast<const float4*>(a.rope_sin + static_cast<int64_t>(pos) * half + pair0);
      const float cs[4] = {c4.x, c4.y, c4.z, c4.w};
      const float sn[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        const float x0 = o[2 * p], x1 = o[2 * p + 1];
        o[2 * p] = x0 * cs[p] - x1 * sn[p];
        o[2 * p + 1] = x0 * sn[p] + x1 * cs[p];
      }
    }
    store8(x + col, o);
  }
}

template <int kGroupLanes>
void launch_rms_lanes(const RmsRopeArgs& a, int chunks, cudaStream_t s) {
  const int blocks = (a.rows * (a.weight2 != nullptr ? 2 : 1) + 7) / 8;
  switch (chunks) {
    case 1: rmsnorm_rope_kernel<1, kGroupLanes><<<blocks, 256, 0, s>>>(a); break;
    case 2: rmsnorm_rope_kernel<2, kGroupLanes><<<blocks, 256, 0, s>>>(a); break;
    case 4: rmsnorm_rope_kernel<4, kGroupLanes><<<blocks, 256, 0, s>>>(a); break;
    case 6: rmsnorm_rope_kernel<6, kGroupLanes><<<blocks, 256, 0, s>>>(a); break;
    case 8: rmsnorm_rope_kernel<8, kGroupLanes><<<blocks, 256, 0, s>>>(a); break;
    case 12: rmsnorm_rope_kernel<12, kGroupLanes><<<blocks, 256, 0, s>>>(a); break;
    case 16: rmsnorm_rope_kernel<16, kGroupLanes><<<blocks, 256, 0, s>>>(a); break;
    default: throw std::runtime_error("rmsnorm_rope: unsupported row width");
  }
}

__global__ void __launch_bounds__(256) sched_step_kernel(SchedStepArgs a) {
  const int64_t n4 = a.n / 4;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float cv[4], uv[4];
    if (a.pred_is_bf16) {
      const uint2 c = reinterpret_cast<const uint2*>(a.cond)[i];
      float2 c0 = unpack_bf16x2(c.x), c1 = unpack_bf16x2(c.y);
      cv[0] = c0.x; cv[1] = c0.y; cv[2] = c1.x; cv[3] = c1.y;
      if (a.uncond) {
        const uint2 u = reinterpret_cast<const uint2*>(a.uncond)[i];
        float2 u0 = unpack_bf16x2(u.x), u1 = unpack_bf16x2(u.y);
        uv[0] = u0.x; uv[1] = u0.y; uv[2] = u1.x; uv[3] = u1.y;
      }
    } else {
      const float4 c = reinterpret_cast<const float4*>(a.cond)[i];
      cv[0] = c.x; cv[1] = c.y; cv[2] = c.z; cv[3] = c.w;
      if (a.uncond) {
        const float4 u = reinterpret_cast<const float4*>(a.uncond)[i];
        uv[0] = u.x; uv[1] = u.y; uv[2] = u.z; uv[3] = u.w;
      }
    }
    const float4 xs = reinterpret_cast<const float4*>(a.sample)[i];
    const float xv[4] = {xs.x, xs.y, xs.z, xs.w};
    float hc[3][4], hp[3][4];
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      if (a.c_hist_ptr[j]) {
        const float4 t = reinterpret_cast<const float4*>(a.c_hist_ptr[j])[i];
        hc[j][0] = t.x; hc[j][1] = t.y; hc[j][2] = t.z; hc[j][3] = t.w;
      } else {
        hc[j][0] = hc[j][1] = hc[j][2] = hc[j][3] = 0.f;
      }
      if (a.p_hist_ptr[j]) {
        const float4 t = reinterpret_cast<const float4*>(a.p_hist_ptr[j])[i];
        hp[j][0] = t.x; hp[j][1] = t.y; hp[j][2] = t.z; hp[j][3] = t.w;
      } else {
        hp[j][0] = hp[j][1] = hp[j][2] = hp[j][3] = 0.f;
      }
    }
    float lv[4] = {0.f, 0.f, 0.f, 0.f};
    if (a.do_corrector) {
      const float4 t = reinterpret_cast<const float4*>(a.last)[i];
      lv[0] = t.x; lv[1] = t.y; lv[2] = t.z; lv[3] = t.w;
    }
    float out[4], x0v[4], xcv[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float v = a.uncond ? uv[e] + a.guidance * (cv[e] - uv[e]) : cv[e];
      const float x0 = xv[e] - a.sigma * v;
      float xc = xv[e];
      if (a.do_corrector) {
        xc = a.c_last * lv[e] + a.c_x0 * x0;
#pragma unroll
        for (int j = 0; j < 3; ++j) xc += a.c_hist[j] * hc[j][e];
      }
      float nx = a.p_x * xc + a.p_x0 * x0 + a.p_v * v;
#pragma unroll
      for (int j = 0; j < 3; ++j) nx += a.p_hist[j] * hp[j][e];
      out[e] = nx;
      x0v[e] = x0;
      xcv[e] = xc;
    }
    reinterpret_cast<float4*>(a.sample)[i] = make_float4(out[0], out[1], out[2], out[3]);
    if (a.x0_out) reinterpret_cast<float4*>(a.x0_out)[i] = make_float4(x0v[0], x0v[1], x0v[2], x0v[3]);
    if (a.last_out) reinterpret_cast<float4*>(a.last_out)[i] = make_float4(xcv[0], xcv[1], xcv[2], xcv[3]);
  }
}

}  // namespace

void launch_layernorm_modulate(const LayerNormArgs& a, cudaStream_t s) {
  if (a.dim % 256 != 0) throw std::runtime_error("layernorm_modulate: dim must be a multiple of 256");
  if ((a.x_stride % 8) || (a.y_stride % 8)) throw std::runtime_error("layernorm_modulate: strides must be x8");
  const int chunks = a.dim / 256;
  const int blocks = (a.rows + 7) / 8;
  switch (chunks) {
    case 1: layernorm_modulate_kernel<1><<<blocks, 256, 0, s>>>(a); break;
    case 2: layernorm_modulate_kernel<2><<<blocks, 256, 0, s>>>(a); break;
    case 4: layernorm_modulate_kernel<4><<<blocks, 256, 0, s>>>(a); break;
    case 6: layernorm_modulate_kernel<6><<<blocks, 256, 0, s>>>(a); break;
    case 8: layernorm_modulate_kernel<8><<<blocks, 256, 0, s>>>(a); break;
    case 12: layernorm_modulate_kernel<12><<<blocks, 256, 0, s>>>(a); break;
    case 16: layernorm_modulate_kernel<16><<<blocks, 256, 0, s>>>(a); break;
    default: throw std::runtime_error("layernorm_modulate: unsupported dim");
  }
}

void launch_rmsnorm_rope(const RmsRopeArgs& a, cudaStream_t s) {
  const int row_width = a.width * a.groups;
  if (row_width % 256 != 0) throw std::runtime_error("rmsnorm_rope: row width must be a multiple of 256");
  if (a.x_stride % 8) throw std::runtime_error("rmsnorm_rope: stride must be x8");
  const int chunks = row_width / 256;
  if (a.groups == 1) {
    launch_rms_lanes<32>(a, chunks, s);
  } else if (a.width == 128) {
    launch_rms_lanes<16>(a, chunks, s);
  } else if (a.width == 64) {
    launch_rms_lanes<8>(a, chunks, s);
  } else {
    throw std::runtime_error("rmsnorm_rope: per-head width must be 64 or 128");
  }
}

void launch_sched_step(const SchedStepArgs& a, cudaStream_t s) {
  if (a.n % 4 != 0) throw std::runtime_error("sched_step: element count must be a multiple of 4");
  const int64_t n4 = a.n / 4;
  int64_t blocks = (n4 + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  if (blocks < 1) blocks = 1;
  sched_step_kernel<<<static_cast<int>(blocks), 256, 0, s>>>(a);
}

}  // namespace ds
