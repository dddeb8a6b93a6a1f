// INT8 transport of the ring-attention key/value chunks over NVSwitch peer memory (sm_100a).
//
// With the codec on, a ring rank does not let its peers read its bf16 K/V chunk in place;
// it quantizes the chunk once and pushes the int8 packet into every ring peer's slot, so
// the bytes that cross NVLink are 132 per (token, head) vector of 128 values instead of 256:
//
//  * ring_quant_push   one warp per (row, part, head) vector of D values (part 0 = K,
//                      1 = V): absolute maximum across the warp, scale = max(amax, 1e-30) /
//                      127, q = clamp(rint(x / scale), -127, 127) with an IEEE division,
//                      and the int8 values plus the fp32 scale stored into slot `src` of
//                      every other ring member's heap (plain 16-byte-granular stores).
//  * ring_dequant      after the ring barrier: each peer slot of this rank's heap becomes a
//                      bf16 buffer laid out like the local receive buffer ([rows, 3w] with K
//                      at column w and V at 2w), which the attention kernel then reads as an
//                      extra key/value source from local memory.
// Slot layout (per source): int8 [rows][2w] (K then V), then fp32 scales [rows][2 * heads].
// The quantisation is symmetric per (token, head) as in the reference's ring codec
// (workers/ditserve/models/wan/ring_quant.py:56-98); the scale is kept in fp32 here.
#include "sm100.cuh"
#include "kernels.h"

namespace ds {
namespace {

template <int D>
__global__ void __launch_bounds__(256) ring_quant_push_kernel(RingCodecArgs a) {
  constexpr int kPer = D / 32;  // values per lane (4 for D = 128, 2 for D = 64)
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int vec_per_row = 2 * a.heads;
  if (warp >= static_cast<int64_t>(a.rows) * vec_per_row) return;
  const int row = static_cast<int>(warp / vec_per_row);
  const int vec = static_cast<int>(warp - static_cast<int64_t>(row) * vec_per_row);  // part * heads + head
  const int width = a.heads * D;
  const __nv_bfloat16* src = reinterpret_cast<const __nv_bfloat16*>(a.kv) + static_cast<int64_t>(row) * a.kv_stride +
                             vec * D + lane * kPer;
  float x[kPer];
  if constexpr (kPer == 4) {
    const uint2 u = *reinterpret_cast<const uint2*>(src);
    const float2 f0 = unpack_bf16x2(u.x), f1 = unpack_bf16x2(u.y);
    x[0] = f0.x;
    x[1] = f0.y;
    x[2] = f1.x;
    x[3] = f1.y;
  } else {
    const float2 f0 = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(src));
    x[0] = f0.x;
    x[1] = f0.y;
  }
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < kPer; ++i) amax = fmaxf(amax, fabsf(x[i]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float scale = fmaxf(amax, 1e-30f) / 127.0f;
  uint32_t packed = 0;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const float q = fminf(fmaxf(rintf(__fdiv_rn(x[i], scale)), -127.f), 127.f);
    packed |= (static_cast<uint32_t>(static_cast<int>(q)) & 0xffu) << (8 * i);
  }
  const int64_t q_off = a.slot_off + static_cast<int64_t>(a.src) * a.slot_bytes +
                        static_cast<int64_t>(row) * (2 * width) + vec * D + lane * kPer;
  const int64_t s_off = a.slot_off + static_cast<int64_t>(a.src) * a.slot_bytes +
                        static_cast<int64_t>(a.rows) * (2 * width) +
                        (static_cast<int64_t>(row) * vec_per_row + vec) * 4;
#pragma unroll 1
  for (int p = 0; p < a.group.size; ++p) {
    if (p == a.group.rank) continue;
    uint8_t* base = reinterpret_cast<uint8_t*>(a.group.base[p]);
    if constexpr (kPer == 4) {
      *reinterpret_cast<uint32_t*>(base + q_off) = packed;
    } else {
      *reinterpret_cast<uint16_t*>(base + q_off) = static_cast<uint16_t>(packed);
    }
    if (lane == 0) *reinterpret_cast<float*>(base + s_off) = scale;
  }
}

// One thread per 16 int8 values of one source slot.
__global__ void __launch_bounds__(256) ring_dequant_kernel(RingCodecArgs a, int src, __nv_bfloat16* out,
                                                           int64_t out_stride) {
  const int width = a.heads * a.head_dim;
  const int64_t per_row = (2 * width) / 16;
  const int64_t n = static_cast<int64_t>(a.rows) * per_row;
  const uint8_t* slot = reinterpret_cast<const uint8_t*>(a.group.base[a.group.rank]) + a.slot_off +
                        static_cast<int64_t>(src) * a.slot_bytes;
  const float* scales = reinterpret_cast<const float*>(slot + static_cast<int64_t>(a.rows) * (2 * width));
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = i / per_row;
    const int col = static_cast<int>(i - row * per_row) * 16;  // column in [0, 2w)
    const uint4 q = *reinterpret_cast<const uint4*>(slot + row * (2 * width) + col);
    const float s = scales[row * (2 * a.heads) + col / a.head_dim];
    const uint32_t w4[4] = {q.x, q.y, q.z, q.w};
    uint32_t o[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int b0 = static_cast<int8_t>(w4[j] & 0xffu), b1 = static_cast<int8_t>((w4[j] >> 8) & 0xffu);
      const int b2 = static_cast<int8_t>((w4[j] >> 16) & 0xffu), b3 = static_cast<int8_t>(w4[j] >> 24);
      o[2 * j] = pack_bf16x2(static_cast<float>(b0) * s, static_cast<float>(b1) * s);
      o[2 * j + 1] = pack_bf16x2(static_cast<float>(b2) * s, static_cast<float>(b3) * s);
    }
    // K (col < w) goes to column w of the [rows, 3w] layout, V to column 2w
    __nv_bfloat16* dst = out + row * out_stride + width + col;
    reinterpret_cast<uint4*>(dst)[0] = make_uint4(o[0], o[1], o[2], o[3]);
    reinterpret_cast<uint4*>(dst)[1] = make_uint4(o[4], o[5], o[6], o[7]);
  }
}

}  // namespace

int64_t ring_slot_bytes(int rows, int heads, int head_dim) {
  const int64_t q = static_cast<int64_t>(rows) * 2 * heads * head_dim;
  const int64_t s = static_cast<int64_t>(rows) * 2 * heads * 4;
  return (q + s + 255) / 256 * 256;
}

void launch_ring_quant_push(const RingCodecArgs& a, cudaStream_t s) {
  if (a.head_dim != 64 && a.head_dim != 128) throw std::runtime_error("ring codec: head_dim must be 64 or 128");
  if (a.kv_stride % 8 != 0 || reinterpret_cast<uintptr_t>(a.kv) % 16 != 0)
    throw std::runtime_error("ring codec: 16-byte aligned K/V rows required");
  if (a.slot_off % 256 != 0 || a.slot_bytes < ring_slot_bytes(a.rows, a.heads, a.head_dim))
    throw std::runtime_error("ring codec: slot too small or misaligned");
  const int64_t warps = static_cast<int64_t>(a.rows) * 2 * a.heads;
  const int64_t blocks = (warps * 32 + 255) / 256;
  if (blocks <= 0) return;
  if (a.head_dim == 128)
    ring_quant_push_kernel<128><<<static_cast<unsigned>(blocks), 256, 0, s>>>(a);
  else
    ring_quant_push_kernel<64><<<static_cast<unsigned>(blocks), 256, 0, s>>>(a);
}

void launch_ring_dequant(const RingCodecArgs& a, int src, void* out, int64_t out_stride, cudaStream_t s) {
  if (src < 0 || src >= a.group.size || src == a.group.rank) throw std::runtime_error("ring codec: bad source slot");
  if (out_stride % 8 != 0 || reinterpret_cast<uintptr_t>(out) % 16 != 0)
    throw std::runtime_error("ring codec: 16-byte aligned output rows required");
  const int64_t n = static_cast<int64_t>(a.rows) * (2 * a.heads * a.head_dim) / 16;
  int64_t blocks = (n + 255) / 256;
  if (blocks > 148 * 8) blocks = 148 * 8;
  if (blocks <= 0) return;
  ring_dequant_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(a, src, reinterpret_cast<__nv_bfloat16*>(out),
                                                                    out_stride);
}

}  // namespace ds
