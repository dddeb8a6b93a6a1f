// Fused compute + collective kernels over NVSwitch peer memory (sm_100a).
//
// Every buffer a peer touches lives in a symmetric heap: one cudaMalloc per
// process, exported with a CUDA IPC handle and opened by every other rank, so
// a kernel holds plain device pointers into its peers' memory and moves data
// with ordinary 16-byte loads/stores over NVLink (no TMA multicast anywhere).
//
// Synchronisation uses monotonically increasing 64-bit epochs in per-channel
// flag arrays at the head of each heap: rank r signals rank s by a system-scope
// release store of the epoch into s's flags[channel][r]; a waiter acquires
// until its own slot reaches the epoch.  Every wait is bounded by a %globaltimer
// limit; on expiry the kernel records kStatusPeerTimeout in the status word and
// returns instead of hanging (no trap).
//
//  * group_barrier       one warp: signal all peers, wait for all peers.
//  * cfg_step_peer       CFG pair: signal partner, wait, then read the partner's
//                        prediction over NVLink and apply guidance + the UniPC /
//                        Euler latent update in one pass (reference: exchange_predictions
//                        all_gather + combine + scheduler.step,
//                        workers/ditserve/models/xdit/wan.py:187-203, block.py:472-486).
//  * qkv_scatter         Ulysses input all-to-all fused with RMS qk-norm (across heads)
//                        and RoPE: each warp normalises one token's q/k, rotates them and
//                        stores every head group directly into the owning rank's receive
//                        buffer (reference: usp.py:207-270 + transformer_wan.py:158-191).
//  * allgather_rows      sequence all-gather by peer stores (SP output gather, usp K12).
//  * group_flag          doorbell stop flag MAX over an SP group in one launch: the flag
//                        rides in the low bit of the barrier epoch (reference: all_reduce MAX
//                        of an int, workers/ditserve/models/xdit/wan.py:257-271).
//  * put_peers           16-byte vector copy of one buffer into several members' heaps
//                        (regroup state broadcast; reference: host-staged packet file +
//                        block_import, study.cpp:1395-1411, parallel.py:903-1050).
// The inverse (head->sequence) all-to-all is fused into the attention epilogue
// (attention.cu, peer-store mode).
#include "sm100.cuh"
#include "kernels.h"

namespace ds {
namespace {

__device__ __forceinline__ void st_release_sys(uint64_t* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// wait until *p >= epoch; false on timeout (status recorded)
__device__ __forceinline__ bool wait_flag(const uint64_t* p, uint64_t epoch, unsigned long long limit_ns, int* status,
                                          int where) {
  if (ld_acquire_sys(p) >= epoch) return true;
  const unsigned long long t0 = globaltimer_ns();
  while (true) {
    for (int i = 0; i < 32; ++i)
      if (ld_acquire_sys(p) >= epoch) return true;
    if (globaltimer_ns() - t0 > limit_ns) {
      report_status(status, kStatusPeerTimeout, where);
      return false;
    }
  }
}

// lanes 0..P-1 each own one peer
__device__ __forceinline__ bool warp_barrier(const PeerGroup& g, int channel, uint64_t epoch, int* status, int where) {
  const int lane = threadIdx.x & 31;
  __threadfence_system();
  __syncwarp();
  bool ok = true;
  if (lane < g.size && lane != g.rank) {
    uint64_t* remote = g.flags[lane] + channel * kMaxPeers + g.rank;
    st_release_sys(remote, epoch);
  }
  __syncwarp();
  if (lane < g.size && lane != g.rank) {
    const uint64_t* mine = g.flags[g.rank] + channel * kMaxPeers + lane;
    ok = wait_flag(mine, epoch, g.timeout_ns, status, where);
  }
  return __all_sync(0xffffffffu, ok);
}

__global__ void group_barrier_kernel(PeerGroup g, int channel, uint64_t epoch, int* status) {
  warp_barrier(g, channel, epoch, status, 300 + channel);
}

// ---------------------------------------------------------------------------
// CFG exchange + guidance + latent update.  Every block signals the partner (the
// same epoch, an idempotent release store) and then waits for the partner's
// signal before it reads the partner's prediction.  No block depends on another
// block of its own grid, so the exchange completes whatever subset of the grid
// happens to be resident on either GPU.
__global__ void __launch_bounds__(256) cfg_step_peer_kernel(SchedStepArgs a, PeerGroup g, int channel,
                                                            uint64_t epoch, const void* mine, int64_t theirs_off,
                                                            int my_role, int* status) {
  __shared__ int ok_s;
  if (threadIdx.x < 32) {
    const bool ok = warp_barrier(g, channel, epoch, status, 320);
    if (threadIdx.x == 0) ok_s = ok ? 1 : 0;
  }
  __syncthreads();
  if (!ok_s) return;
  const int partner = 1 - g.rank;
  const uint8_t* theirs = reinterpret_cast<const uint8_t*>(g.base[partner]) + theirs_off;
  const void* cond = my_role == 0 ? mine : theirs;
  const void* uncond = my_role == 0 ? static_cast<const void*>(theirs) : mine;
  const int64_t n4 = a.n / 4;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float cv[4], uv[4];
    const uint2 c = reinterpret_cast<const uint2*>(cond)[i];
    const uint2 u = reinterpret_cast<const uint2*>(uncond)[i];
    float2 c0 = unpack_bf16x2(c.x), c1 = unpack_bf16x2(c.y), u0 = unpack_bf16x2(u.x), u1 = unpack_bf16x2(u.y);
    cv[0] = c0.x; cv[1] = c0.y; cv[2] = c1.x; cv[3] = c1.y;
    uv[0] = u0.x; uv[1] = u0.y; uv[2] = u1.x; uv[3] = u1.y;
    const float4 xs = reinterpret_cast<const float4*>(a.sample)[i];
    const float xv[4] = {xs.x, xs.y, xs.z, xs.w};
    float hc[3][4], hp[3][4], lv[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      const float4 t1 = a.c_hist_ptr[j] ? reinterpret_cast<const float4*>(a.c_hist_ptr[j])[i] : make_float4(0, 0, 0, 0);
      const float4 t2 = a.p_hist_ptr[j] ? reinterpret_cast<const float4*>(a.p_hist_ptr[j])[i] : make_float4(0, 0, 0, 0);
      hc[j][0] = t1.x; hc[j][1] = t1.y; hc[j][2] = t1.z; hc[j][3] = t1.w;
      hp[j][0] = t2.x; hp[j][1] = t2.y; hp[j][2] = t2.z; hp[j][3] = t2.w;
    }
    if (a.do_corrector) {
      const float4 t = reinterpret_cast<const float4*>(a.last)[i];
      lv[0] = t.x; lv[1] = t.y; lv[2] = t.z; lv[3] = t.w;
    }
    float out[4], x0v[4], xcv[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float v = uv[e] + a.guidance * (cv[e] - uv[e]);
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
    if (a.delta_out)
      reinterpret_cast<float4*>(a.delta_out)[i] =
          make_float4(cv[0] - uv[0], cv[1] - uv[1], cv[2] - uv[2], cv[3] - uv[3]);
    if (a.x0_out) reinterpret_cast<float4*>(a.x0_out)[i] = make_float4(x0v[0], x0v[1], x0v[2], x0v[3]);
    if (a.last_out) reinterpret_cast<float4*>(a.last_out)[i] = make_float4(xcv[0], xcv[1], xcv[2], xcv[3]);
  }
}

// ---------------------------------------------------------------------------
__device__ __forceinline__ void load8f(const __nv_bfloat16* p, float (&f)[8]) {
  uint4 u = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = unpack_bf16x2(w[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}
__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = unpack_bf16x2(w[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint4 u;
  u.x = pack_bf16x2(f[0], f[1]);
  u.y = pack_bf16x2(f[2], f[3]);
  u.z = pack_bf16x2(f[4], f[5]);
  u.w = pack_bf16x2(f[6], f[7]);
  return u;
}

// One warp per local token row of qkv [B*Sl, 3*H*D].  kChunks = H*D / 256.
// Destination on rank j: recv[(b*S + rank*Sl + t) * 3*Hl*D + part*Hl*D + (h - j*Hl)*D + d].
// The warp issues the loads of all three parts (q, k, v) before any arithmetic (widths up to
// 1536: 3 x kChunks 16-byte loads per lane kept as raw bf16), so a token's whole 3*H*D row is
// in flight at once; the kernel is bound by HBM latency otherwise (one part in flight).  v is
// stored as loaded.
template <int kChunks>
__global__ void __launch_bounds__(128) qkv_scatter_kernel(QkvScatterArgs a) {
  constexpr int kPre = kChunks <= 6 ? 3 : 1;  // parts whose loads are issued up front
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= a.rows) return;
  const int width = a.heads * a.head_dim;  // H*D
  const int hl_width = width / a.group.size;  // Hl*D
  const int b = warp / a.seq_local;
  const int t = warp - b * a.seq_local;
  const int64_t dst_row = static_cast<int64_t>(b) * a.seq_local * a.group.size + a.group.rank * a.seq_local + t;
  const __nv_bfloat16* src = reinterpret_cast<const __nv_bfloat16*>(a.qkv) + static_cast<int64_t>(warp) * a.qkv_stride;
  const int half = a.head_dim / 2;
  uint4 raw[kPre][kChunks];
#pragma unroll
  for (int p = 0; p < kPre; ++p)
#pragma unroll
    for (int c = 0; c < kChunks; ++c)
      raw[p][c] = *reinterpret_cast<const uint4*>(src + p * width + c * 256 + lane * 8);
#pragma unroll
  for (int part = 0; part < 3; ++part) {
    uint4(&r)[kChunks] = raw[kPre == 3 ? part : 0];
    if (kPre == 1 && part > 0) {
#pragma unroll
      for (int c = 0; c < kChunks; ++c)
        r[c] = *reinterpret_cast<const uint4*>(src + part * width + c * 256 + lane * 8);
    }
    if (part < 2) {
      // RMS across all heads of the token, weight, bf16 rounding, then RoPE.  Same
      // summation order as rmsnorm_rope_kernel (per-chunk partials), so the fused and the
      // unfused paths produce bit-identical q/k.
      float ss = 0.f;
#pragma unroll
      for (int c = 0; c < kChunks; ++c) {
        float v[8];
        unpack8(r[c], v);
        float cs = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) cs += v[i] * v[i];
        ss += cs;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      const float rs = rsqrtf(ss / static_cast<float>(width) + a.eps);
      const __nv_bfloat16* w = reinterpret_cast<const __nv_bfloat16*>(part == 0 ? a.wq : a.wk);
      const int pos = a.pos_base + t + a.group.rank * a.seq_local;  // global position in the sequence
#pragma unroll
      for (int c = 0; c < kChunks; ++c) {
        const int col = c * 256 + lane * 8;
        float v[8], wv[8];
        unpack8(r[c], v);
        load8f(w + col, wv);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = __bfloat162float(__float2bfloat16_rn(v[i] * rs * wv[i]));
        if (a.rope_cos != nullptr) {
          const int pair0 = (col % a.head_dim) / 2;
          const float4 c4 = *reinterpret_cast<const float4*>(a.rope_cos + static_cast<int64_t>(pos) * half + pair0);
          const float4 s4 = *reinterpret_cast<const float4*>(a.rope_sin + static_cast<int64_t>(pos) * half + pair0);
          const float cs[4] = {c4.x, c4.y, c4.z, c4.w};
          const float sn[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
          for (int p = 0; p < 4; ++p) {
            const float x0 = v[2 * p], x1 = v[2 * p + 1];
            v[2 * p] = x0 * cs[p] - x1 * sn[p];
            v[2 * p + 1] = x0 * sn[p] + x1 * cs[p];
          }
        }
        r[c] = pack8(v);
      }
    }
#pragma unroll
    for (int c = 0; c < kChunks; ++c) {
      const int col = c * 256 + lane * 8;
      const int owner = col / hl_width;
      const int dcol = part * hl_width + (col - owner * hl_width);
      __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(reinterpret_cast<uint8_t*>(a.group.base[owner]) + a.recv_off);
      *reinterpret_cast<uint4*>(dst + dst_row * (3 * hl_width) + dcol) = r[c];
    }
  }
}

// Every rank stores its [rows, cols] slice at row offset rank*rows of every peer's buffer.
__global__ void __launch_bounds__(256) allgather_rows_kernel(PeerGroup g, const uint4* src, int64_t n16,
                                                             int64_t dst_off, int64_t slice16) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n16;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint4 v = src[i];
#pragma unroll 1
    for (int p = 0; p < g.size; ++p) {
      uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(g.base[p]) + dst_off);
      dst[g.rank * slice16 + i] = v;
    }
  }
}

// Copy a strided 4-D slice (elements of `esize` bytes) into a contiguous buffer of one
// group member (halo exchange of the patch-parallel VAE: a boundary row/column of this
// rank's feature map lands directly in the neighbour's halo buffer).
__global__ void __launch_bounds__(256) strided_put_kernel(PeerGroup g, int peer, const uint8_t* src, StridedSlice sl,
                                                          int64_t dst_off) {
  const int64_t n = static_cast<int64_t>(sl.size[0]) * sl.size[1] * sl.size[2] * sl.size[3];
  uint8_t* dst = reinterpret_cast<uint8_t*>(g.base[peer]) + dst_off;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    int64_t r = i;
    const int64_t i3 = r % sl.size[3];
    r /= sl.size[3];
    const int64_t i2 = r % sl.size[2];
    r /= sl.size[2];
    const int64_t i1 = r % sl.size[1];
    const int64_t i0 = r / sl.size[1];
    const uint8_t* s = src + i0 * sl.stride[0] + i1 * sl.stride[1] + i2 * sl.stride[2] + i3 * sl.stride[3];
    if (sl.esize == 2) {
      reinterpret_cast<uint16_t*>(dst)[i] = *reinterpret_cast<const uint16_t*>(s);
    } else {
      reinterpret_cast<uint32_t*>(dst)[i] = *reinterpret_cast<const uint32_t*>(s);
    }
  }
}

// Lane p signals peer p with 2*epoch + flag and waits for 2*epoch from every peer; the
// OR of the low bits is the group's MAX of a 0/1 flag.  Callers alternate between two
// channels by epoch parity: a peer can reach epoch+2 on this channel only after this
// rank signalled epoch+1 on the other one, i.e. after it has read this epoch's value.
__global__ void group_flag_kernel(PeerGroup g, int channel, uint64_t epoch, int flag, int* out, int* status) {
  const int lane = threadIdx.x & 31;
  const uint64_t mine_v = 2 * epoch + (flag ? 1u : 0u);
  __threadfence_system();
  if (lane < g.size && lane != g.rank) st_release_sys(g.flags[lane] + channel * kMaxPeers + g.rank, mine_v);
  __syncwarp();
  bool ok = true;
  int f = (lane == g.rank) ? (flag ? 1 : 0) : 0;
  if (lane < g.size && lane != g.rank) {
    const uint64_t* slot = g.flags[g.rank] + channel * kMaxPeers + lane;
    ok = wait_flag(slot, 2 * epoch, g.timeout_ns, status, 340 + channel);
    if (ok) f = static_cast<int>(ld_acquire_sys(slot) & 1u);
  }
  const bool all_ok = __all_sync(0xffffffffu, ok);
  const int any = __any_sync(0xffffffffu, f != 0);
  if (lane == 0) *out = all_ok ? any : -1;
}

__global__ void __launch_bounds__(256) put_peers_kernel(PeerGroup g, unsigned mask, const uint4* src, int64_t n16,
                                                        int64_t dst_off) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n16;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint4 v = src[i];
#pragma unroll 1
    for (int p = 0; p < g.size; ++p) {
      if (!((mask >> p) & 1u)) continue;
      reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(g.base[p]) + dst_off)[i] = v;
    }
  }
}

}  // namespace

void launch_group_flag(const PeerGroup& g, int channel, uint64_t epoch, int flag, int* out, int* status,
                       cudaStream_t s) {
  if (g.size < 1 || g.size > kMaxPeers || channel < 0 || channel >= kChannels) throw std::runtime_error("bad group");
  group_flag_kernel<<<1, 32, 0, s>>>(g, channel, epoch, flag, out, status);
}

void launch_put_peers(const PeerGroup& g, unsigned mask, const void* src, int64_t bytes, int64_t dst_off,
                      cudaStream_t s) {
  if (bytes % 16 != 0 || dst_off % 16 != 0 || reinterpret_cast<uintptr_t>(src) % 16 != 0)
    throw std::runtime_error("put_peers: 16-byte aligned source, size and offset required");
  if (mask >> g.size) throw std::runtime_error("put_peers: mask names ranks outside the group");
  const int64_t n16 = bytes / 16;
  if (n16 == 0 || mask == 0) return;
  int64_t blocks = (n16 + 255) / 256;
  if (blocks > 148 * 4) blocks = 148 * 4;
  put_peers_kernel<<<static_cast<int>(blocks), 256, 0, s>>>(g, mask, reinterpret_cast<const uint4*>(src), n16,
                                                            dst_off);
}

void launch_strided_put(const PeerGroup& g, int peer, const void* src, const StridedSlice& sl, int64_t dst_off,
                        cudaStream_t s) {
  if (peer < 0 || peer >= g.size) throw std::runtime_error("strided_put: peer outside the group");
  if (sl.esize != 2 && sl.esize != 4) throw std::runtime_error("strided_put: element size must be 2 or 4");
  const int64_t n = static_cast<int64_t>(sl.size[0]) * sl.size[1] * sl.size[2] * sl.size[3];
  if (n <= 0) return;
  int64_t blocks = (n + 255) / 256;
  if (blocks > 148 * 8) blocks = 148 * 8;
  strided_put_kernel<<<static_cast<int>(blocks), 256, 0, s>>>(g, peer, reinterpret_cast<const uint8_t*>(src), sl,
                                                              dst_off);
}

void launch_group_barrier(const PeerGroup& g, int channel, uint64_t epoch, int* status, cudaStream_t s) {
  if (g.size < 1 || g.size > kMaxPeers || channel < 0 || channel >= kChannels) throw std::runtime_error("bad group");
  group_barrier_kernel<<<1, 32, 0, s>>>(g, channel, epoch, status);
}

void launch_cfg_step_peer(const SchedStepArgs& a, const PeerGroup& g, int channel, uint64_t epoch, const void* mine,
                          int64_t theirs_off, int my_role, int* status, cudaStream_t s) {
  if (g.size != 2) throw std::runtime_error("cfg_step_peer needs a group of two");
  if (a.n % 4 != 0) throw std::runtime_error("cfg_step_peer: element count must be a multiple of 4");
  int64_t blocks = (a.n / 4 + 255) / 256;
  if (blocks > 148 * 8) blocks = 148 * 8;
  if (blocks < 1) blocks = 1;
  cfg_step_peer_kernel<<<static_cast<int>(blocks), 256, 0, s>>>(a, g, channel, epoch, mine, theirs_off, my_role,
                                                                status);
}

void launch_qkv_scatter(const QkvScatterArgs& a, cudaStream_t s) {
  const int width = a.heads * a.head_dim;
  if (width % 256 != 0 || (width / a.group.size) % 8 != 0 || a.heads % a.group.size != 0)
    throw std::runtime_error("qkv_scatter: heads*head_dim must be a multiple of 256 and split over the group");
  const int chunks = width / 256;
  // four warps (tokens) per block: at 100-200 registers a thread, small blocks keep 12-16
  // warps resident per SM
  const int blocks = (a.rows + 3) / 4;
  switch (chunks) {
    case 2: qkv_scatter_kernel<2><<<blocks, 128, 0, s>>>(a); break;
    case 4: qkv_scatter_kernel<4><<<blocks, 128, 0, s>>>(a); break;
    case 6: qkv_scatter_kernel<6><<<blocks, 128, 0, s>>>(a); break;
    case 8: qkv_scatter_kernel<8><<<blocks, 128, 0, s>>>(a); break;
    case 12: qkv_scatter_kernel<12><<<blocks, 128, 0, s>>>(a); break;
    default: throw std::runtime_error("qkv_scatter: unsupported width");
  }
}

void launch_allgather_rows(const PeerGroup& g, const void* src, int64_t bytes, int64_t dst_off, cudaStream_t s) {
  if (bytes % 16 != 0 || dst_off % 16 != 0) throw std::runtime_error("allgather_rows: 16-byte multiples required");
  const int64_t n16 = bytes / 16;
  int64_t blocks = (n16 + 255) / 256;
  if (blocks > 148 * 4) blocks = 148 * 4;
  if (blocks < 1) blocks = 1;
  allgather_rows_kernel<<<static_cast<int>(blocks), 256, 0, s>>>(g, reinterpret_cast<const uint4*>(src), n16,
                                                                  dst_off, n16);
}

}  // namespace ds
