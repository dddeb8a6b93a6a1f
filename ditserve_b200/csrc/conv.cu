// Implicit-GEMM convolution on the 5th-generation tensor cores (sm_100a), channels-last.
//
//   X : [T_in, H_in, W_in, C_in] bf16 (C contiguous)
//   Wt: [C_out_pad, KT * KH * KW * C_in] bf16 (tap-major, then C_in: K contiguous per output channel)
//   Y : [T_out, H_out, W_out, C_out] bf16 = conv(X) + bias (+ R)
//
// Time is "valid" (T_out = T_in - KT + 1: the causal padding, i.e. the cached frames, is in X
// already); space is padded by pad_h / pad_w zeros through TMA out-of-bounds fill, so no padded
// copy of X is ever made.  With pad_h = 0 the caller's X carries its own halo rows, which is how
// patch parallelism feeds the kernel: each neighbour stores its boundary rows straight into this
// rank's X (peer-memory stores) and the conv reads local memory only.
//
// GEMM view: M = output pixels, N = C_out, K = taps x C_in.  One CTA per SM walks 128-pixel x BN
// tiles; a pixel tile is a 32-wide x 4-high block of one output frame, so each K step is one TMA
// box [32 channels, 32 w, 4 h, 1 t] at the tap's offset (64-byte rows, 64-byte swizzle) and one
// box [32 k, BN rows] of the weights.  Warp 0 streams the boxes through a STAGES-deep ring, warp
// 1 issues tcgen05.mma (M = 128, N = BN, K = 16) into one of two TMEM accumulators, and warps
// 2..9 drain the other one through the bias / residual epilogue, as in gemm.cu.
//
// Replaces cuDNN's conv3d / conv2d in the Wan VAE decoder (the reference decodes with
// diffusers' AutoencoderKLWan, distvae-parallelised: workers/xfuser/model_executor/pipelines/
// base_pipeline.py:61,133).
#include "sm100.cuh"
#include "tma_host.h"
#include "kernels.h"

namespace ds {
namespace {

constexpr int kCBM = 128;            // output pixels per tile
constexpr int kCBW = 32, kCBH = 4;   // pixel tile: 32 wide x 4 high
constexpr int kCBK = 32;             // input channels per K step (64-byte rows)
constexpr int kCEpiWarps = 8;
constexpr int kCThreads = 64 + 32 * kCEpiWarps;

template <int BN>
struct ConvCfg {
  static constexpr int kStages = BN <= 128 ? 10 : 8;
  static constexpr int kABytes = kCBM * kCBK * 2;   // 8 KB
  static constexpr int kBBytes = BN * kCBK * 2;
  static constexpr int kAccCols = BN <= 32 ? 32 : BN <= 64 ? 64 : BN <= 128 ? 128 : 256;
  static constexpr int kTmemCols = 2 * kAccCols;
  static constexpr int kSmemBytes = kStages * (kABytes + kBBytes) + 1024 + 256;
};

struct ConvParams {
  int T_out, H_out, W_out, C_in, C_out, C_out_pad;
  int KT, KH, KW, pad_h, pad_w;
  __nv_bfloat16* Y;
  const __nv_bfloat16* bias;  // [C_out_pad] or null
  const __nv_bfloat16* R;     // residual, same layout as Y, or null
  int* status;
};

// UMMA shared-memory descriptor for K-major tiles with 64-byte rows and 64-byte swizzle:
// 8-row groups 512 bytes apart.
__device__ __forceinline__ uint64_t umma_desc_sw64(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr & 0x3FFFF) >> 4);
  d |= static_cast<uint64_t>(1) << 16;            // leading offset (unused by swizzled K-major)
  d |= static_cast<uint64_t>(512 >> 4) << 32;     // stride between 8-row groups
  d |= 1ull << 46;
  d |= 4ull << 61;                                // 64-byte swizzle
  return d;
}

__device__ __forceinline__ void tma_load_4d(void* smem_dst, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
      "[%6];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
      : "memory");
}

template <int BN, bool kRes>
__global__ void __launch_bounds__(kCThreads, 1)
    conv_igemm_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW, ConvParams p) {
  using Cfg = ConvCfg<BN>;
  constexpr int ST = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + ST * Cfg::kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + ST * Cfg::kBBytes);
  uint64_t* empty = full + ST;
  uint64_t* acc_full = empty + ST;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tiles_w = (p.W_out + kCBW - 1) / kCBW;
  const int tiles_h = (p.H_out + kCBH - 1) / kCBH;
  const int tiles_m = p.T_out * tiles_h * tiles_w;
  const int tiles_n = p.C_out_pad / BN;
  const int num_tiles = tiles_m * tiles_n;
  const int cblocks = p.C_in / kCBK;
  const int num_k = p.KT * p.KH * p.KW * cblocks;

  if (threadIdx.x == 0) {
    for (int i = 0; i < ST; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 32 * kCEpiWarps);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmX);
    tma_prefetch_desc(&tmW);
  }
  if (warp == 1) tmem_alloc<Cfg::kTmemCols>(tmem_slot);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  auto tile_origin = [&](int tile, int& t, int& h0, int& w0, int& n0) {
    const int mt = tile / tiles_n;
    n0 = (tile - mt * tiles_n) * BN;
    t = mt / (tiles_h * tiles_w);
    const int r = mt - t * (tiles_h * tiles_w);
    h0 = (r / tiles_w) * kCBH;
    w0 = (r - (r / tiles_w) * tiles_w) * kCBW;
  };

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      int stage = 0;
      uint32_t phase = 0;
      for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
        int t, h0, w0, n0;
        tile_origin(tile, t, h0, w0, n0);
        int kidx = 0;
        for (int kt = 0; kt < p.KT; ++kt)
          for (int kh = 0; kh < p.KH; ++kh)
            for (int kw = 0; kw < p.KW; ++kw)
              for (int cb = 0; cb < cblocks; ++cb, ++kidx) {
                if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, p.status, 50)) goto producer_done;
                mbar_arrive_expect_tx(&full[stage], Cfg::kABytes + Cfg::kBBytes);
                tma_load_4d(sA + stage * Cfg::kABytes, &tmX, cb * kCBK, w0 + kw - p.pad_w, h0 + kh - p.pad_h, t + kt,
                            &full[stage]);
                tma_load_2d(sB + stage * Cfg::kBBytes, &tmW, kidx * kCBK, n0, &full[stage]);
                if (++stage == ST) {
                  stage = 0;
                  phase ^= 1;
                }
              }
      }
    producer_done:;
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      constexpr uint32_t idesc = umma_idesc_bf16(kCBM, BN, false);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1, abort_flag, p.status, 51)) goto mma_done;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * Cfg::kAccCols;
        for (int kb = 0; kb < num_k; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, p.status, 52)) goto mma_done;
          tc_fence_after();
          const uint64_t da = umma_desc_sw64(smem_u32(sA + stage * Cfg::kABytes));
          const uint64_t db = umma_desc_sw64(smem_u32(sB + stage * Cfg::kBBytes));
#pragma unroll
          for (int k = 0; k < kCBK / 16; ++k) umma_bf16_ss(d_tmem, da + 2 * k, db + 2 * k, idesc, (kb | k) != 0);
          umma_commit(&empty[stage]);
          if (++stage == ST) {
            stage = 0;
            phase ^= 1;
          }
        }
        umma_commit(&acc_full[acc]);
      }
    mma_done:;
    }
  } else {
    // ---------------- epilogue warps 2..9: one pixel per TMEM lane ----------------
    const int quarter = warp & 3;
    const int m_local = quarter * 32 + lane;
    const int col_half = (warp - 2) / 4;
    constexpr int kChunks = BN / 32;
    const int c_begin = col_half * ((kChunks + 1) / 2);
    const int c_end = col_half == 0 ? (kChunks + 1) / 2 : kChunks;
    int local = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      int t, h0, w0, n0;
      tile_origin(tile, t, h0, w0, n0);
      if (!mbar_wait(&acc_full[acc], acc_phase, abort_flag, p.status, 53)) break;
      tc_fence_after();
      const int h = h0 + m_local / kCBW;
      const int w = w0 + (m_local % kCBW);
      const bool pix_ok = h < p.H_out && w < p.W_out;
      const int64_t pix = (static_cast<int64_t>(t) * p.H_out + h) * p.W_out + w;
#pragma unroll 1
      for (int c = c_begin; c < c_end; ++c) {
        const int n = n0 + c * 32;
        uint32_t r[32];
        tmem_ld32(tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * Cfg::kAccCols + c * 32, r);
        tmem_wait_ld();
        if (!pix_ok || n >= p.C_out) continue;
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
        if (p.bias != nullptr) {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] += __bfloat162float(p.bias[n + j]);
        }
        __nv_bfloat16* y = p.Y + pix * p.C_out + n;
        if (n + 32 <= p.C_out && (p.C_out & 7) == 0) {
          if (kRes) {
            const uint4* rp = reinterpret_cast<const uint4*>(p.R + pix * p.C_out + n);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const uint4 rv = rp[q];
              const uint32_t rw[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                const float2 f = unpack_bf16x2(rw[u]);
                v[q * 8 + u * 2] += f.x;
                v[q * 8 + u * 2 + 1] += f.y;
              }
            }
          }
          uint4* yp = reinterpret_cast<uint4*>(y);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 o;
            o.x = pack_bf16x2(v[q * 8 + 0], v[q * 8 + 1]);
            o.y = pack_bf16x2(v[q * 8 + 2], v[q * 8 + 3]);
            o.z = pack_bf16x2(v[q * 8 + 4], v[q * 8 + 5]);
            o.w = pack_bf16x2(v[q * 8 + 6], v[q * 8 + 7]);
            yp[q] = o;
          }
        } else {
          // ragged channel tail (an output width that is not a multiple of 32, e.g. RGB)
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            if (n + j < p.C_out) {
              float o = v[j];
              if (kRes) o += __bfloat162float(p.R[pix * p.C_out + n + j]);
              y[j] = __float2bfloat16_rn(o);
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[acc]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (*abort_flag && threadIdx.x == 0) {
    const unsigned long long t0 = globaltimer_ns();
    while (globaltimer_ns() - t0 < 1000000ull) {
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc<Cfg::kTmemCols>(tmem_base);
  }
}

CUtensorMap make_tmap_conv_input(const ConvArgs& a) {
  CUtensorMap map;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(a.C_in), static_cast<cuuint64_t>(a.W_in),
                        static_cast<cuuint64_t>(a.H_in), static_cast<cuuint64_t>(a.T_in)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(a.C_in) * 2, static_cast<cuuint64_t>(a.W_in) * a.C_in * 2,
                           static_cast<cuuint64_t>(a.H_in) * a.W_in * a.C_in * 2};
  cuuint32_t box[4] = {static_cast<cuuint32_t>(kCBK), kCBW, kCBH, 1};
  cuuint32_t elem_strides[4] = {1, 1, 1, 1};
  CUresult r = encode_tiled_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(a.X), dims, strides, box,
                                 elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("conv: input tensor map encode failed: " + std::to_string(int(r)));
  return map;
}

CUtensorMap make_tmap_conv_weight(const ConvArgs& a, int bn) {
  const uint64_t k = static_cast<uint64_t>(a.KT) * a.KH * a.KW * a.C_in;
  CUtensorMap map;
  cuuint64_t dims[2] = {k, static_cast<cuuint64_t>(a.C_out_pad)};
  cuuint64_t strides[1] = {k * 2};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(kCBK), static_cast<cuuint32_t>(bn)};
  cuuint32_t elem_strides[2] = {1, 1};
  CUresult r = encode_tiled_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(a.W), dims, strides, box,
                                 elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("conv: weight tensor map encode failed: " + std::to_string(int(r)));
  return map;
}

template <int BN, bool kRes>
void launch_conv_bn(const ConvArgs& a, cudaStream_t stream) {
  using Cfg = ConvCfg<BN>;
  auto kern = conv_igemm_kernel<BN, kRes>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes);
  const CUtensorMap tmX = make_tmap_conv_input(a);
  const CUtensorMap tmW = make_tmap_conv_weight(a, BN);
  ConvParams p;
  p.T_out = a.T_in - a.KT + 1;
  p.H_out = a.H_in + 2 * a.pad_h - a.KH + 1;
  p.W_out = a.W_in + 2 * a.pad_w - a.KW + 1;
  p.C_in = a.C_in;
  p.C_out = a.C_out;
  p.C_out_pad = a.C_out_pad;
  p.KT = a.KT;
  p.KH = a.KH;
  p.KW = a.KW;
  p.pad_h = a.pad_h;
  p.pad_w = a.pad_w;
  p.Y = reinterpret_cast<__nv_bfloat16*>(a.Y);
  p.bias = reinterpret_cast<const __nv_bfloat16*>(a.bias);
  p.R = reinterpret_cast<const __nv_bfloat16*>(a.R);
  p.status = a.status;
  const int tiles = p.T_out * ((p.H_out + kCBH - 1) / kCBH) * ((p.W_out + kCBW - 1) / kCBW) * (a.C_out_pad / BN);
  const int sms = device_sm_count();
  const int grid = tiles < sms ? tiles : sms;
  if (grid <= 0) return;
  kern<<<grid, kCThreads, Cfg::kSmemBytes, stream>>>(tmX, tmW, p);
}

template <int BN>
void launch_conv_res(const ConvArgs& a, cudaStream_t stream) {
  if (a.R != nullptr)
    launch_conv_bn<BN, true>(a, stream);
  else
    launch_conv_bn<BN, false>(a, stream);
}

}  // namespace

int conv_pick_bn(int c_out_pad) {
  // the widest tile (<= 256 columns, a multiple of 32) that divides the padded output width
  for (int bn : {256, 192, 128, 96, 64, 32})
    if (c_out_pad % bn == 0) return bn;
  return 0;
}

void launch_conv(const ConvArgs& a, cudaStream_t stream) {
  if (a.C_in % kCBK != 0) throw std::runtime_error("conv: C_in must be a multiple of 32");
  if (a.C_out_pad % 32 != 0 || a.C_out > a.C_out_pad) throw std::runtime_error("conv: C_out_pad must be a x32 >= C_out");
  if (a.KT < 1 || a.KH < 1 || a.KW < 1 || a.T_in < a.KT) throw std::runtime_error("conv: bad kernel extent");
  if (a.pad_h < 0 || a.pad_h > 1 || a.pad_w < 0 || a.pad_w > 1) throw std::runtime_error("conv: padding 0 or 1");
  if ((reinterpret_cast<uintptr_t>(a.X) & 15) || (reinterpret_cast<uintptr_t>(a.W) & 15) ||
      (reinterpret_cast<uintptr_t>(a.Y) & 15) || (a.R && (reinterpret_cast<uintptr_t>(a.R) & 15)))
    throw std::runtime_error("conv: tensors must be 16-byte aligned");
  const int bn = a.bn_override > 0 ? a.bn_override : conv_pick_bn(a.C_out_pad);
  switch (bn) {
    case 256: launch_conv_res<256>(a, stream); break;
    case 192: launch_conv_res<192>(a, stream); break;
    case 128: launch_conv_res<128>(a, stream); break;
    case 96: launch_conv_res<96>(a, stream); break;
    case 64: launch_conv_res<64>(a, stream); break;
    case 32: launch_conv_res<32>(a, stream); break;
    default: throw std::runtime_error("conv: unsupported output width");
  }
}

}  // namespace ds
