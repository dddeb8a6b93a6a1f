// Persistent, warp-specialised bf16 GEMM for sm_100a:  C = epilogue(A * B^T)
//
//   A : [M, K] bf16, row-major (activations, K contiguous)
//   B : [N, K] bf16, row-major (nn.Linear weight layout [out, in])
//   C : [M, N] bf16, row-major
//
// One CTA per SM walks output tiles of 128 x BN.  Warp 0 (one lane) streams
// A/B k-blocks of 64 elements into a STAGES-deep shared-memory ring with TMA
// (128-byte swizzle, no multicast).  Warp 1 owns TMEM: it allocates two
// 128 x BN fp32 accumulators and one lane issues tcgen05.mma (M=128, N=BN,
// K=16 per instruction) into one of them while the eight epilogue warps
// (warps 2..9, two per TMEM lane quarter, each taking half the columns) drain the
// other one, so the epilogue of tile i overlaps the main loop of tile i+1.
//
// Epilogues are fused so the hot DiT ops never round-trip through HBM:
//   kEpiNone      C = acc + bias
//   kEpiGelu      C = gelu_tanh(acc + bias)                (FFN up-projection)
//   kEpiGatedRes  C = R + gate[b, n] * (acc + bias)         (adaLN-Zero residual)
//   kEpiRes       C = R + (acc + bias)                      (plain residual)
// gate is fp32 with a per-batch row stride; b = row / rows_per_batch.
// R may alias C (in-place residual update): each element is read and then
// written by the same thread.
//
// Replaces the reference's cuBLAS nn.Linear calls around its attention and
// FFN (workers/xfuser/model_executor/models/transformers/transformer_wan.py:50-69,
// :154; diffusers FeedForward) and the torch elementwise adaLN gating
// (workers/ditserve/models/wan/block.py:282-297).
#include <cstdlib>

#include "sm100.cuh"
#include "tma_host.h"
#include "kernels.h"

namespace ds {
namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kEpiWarps = 8;    // two warps per TMEM lane quarter, each drains half the columns
constexpr int kThreads = 64 + 32 * kEpiWarps;  // warp0 TMA, warp1 MMA, warps 2..9 epilogue

template <int BN>
struct GemmCfg {
  static constexpr int kStages = BN == 256 ? 4 : (BN == 128 ? 6 : 8);
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kTmemCols = 2 * BN;  // two accumulators
  static constexpr int kSmemBytes = kStages * (kABytes + kBBytes) + 1024 /*align*/ + 256 /*barriers*/;
};

struct EpiParams {
  int M, N, K;
  __nv_bfloat16* C;
  int64_t ldc;
  const __nv_bfloat16* bias;
  const __nv_bfloat16* R;
  int64_t ldr;
  const float* gate;
  int64_t gate_stride;
  int rows_per_batch;
  const int* row_batch;
  int* status;
};

// The residual segment of one output row that an epilogue thread drains: kCount chunks of 32
// bf16 starting at column n0 + c_begin * 32.  It is requested before the thread waits for the
// accumulator, so the loads travel while the tile's main loop runs (a short-K GEMM such as the
// gated out-projection otherwise waits for one residual round trip per chunk).
template <int kCount>
struct ResidualRow {
  uint4 v[kCount][4];
};

template <int kCount, int EPI>
__device__ __forceinline__ void prefetch_residual(const EpiParams& p, int m, bool row_ok, int n0, int c_begin,
                                                  ResidualRow<kCount>& rr) {
  if ((EPI == kEpiGatedRes || EPI == kEpiRes) && row_ok) {
    const uint4* rp = reinterpret_cast<const uint4*>(p.R + static_cast<int64_t>(m) * p.ldr + n0 + c_begin * 32);
#pragma unroll
    for (int i = 0; i < kCount; ++i)
#pragma unroll
      for (int q = 0; q < 4; ++q) rr.v[i][q] = rp[i * 4 + q];
  }
}

// Drains accumulator columns [c_begin*32, (c_begin + kCount)*32) of one TMEM lane (row m of the
// output) through the fused epilogue into C.  `taddr` addresses the lane's first accumulator column.
template <int BN, int EPI, int kCount>
__device__ __forceinline__ void epilogue_rows(const EpiParams& p, uint32_t taddr, int m, bool row_ok, int n0,
                                              const float* gate_row, int c_begin, const ResidualRow<kCount>& rr) {
  // gate rows are fp32 [B, N]; 16-byte vector loads when the row allows them
  const bool gate_vec = gate_row != nullptr && (reinterpret_cast<uintptr_t>(gate_row) & 15) == 0;
#pragma unroll
  for (int i = 0; i < kCount; ++i) {
    const int c = c_begin + i;
    const int n = n0 + c * 32;
    uint32_t r[32];
    tmem_ld32(taddr + c * 32, r);
    tmem_wait_ld();
    if (row_ok) {
      float v[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
      if (p.bias != nullptr) {
        const uint4* bp = reinterpret_cast<const uint4*>(p.bias + n);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4 b = __ldg(bp + q);
          const uint32_t bw[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            float2 f = unpack_bf16x2(bw[t]);
            v[q * 8 + t * 2] += f.x;
            v[q * 8 + t * 2 + 1] += f.y;
          }
        }
      }
      if (EPI == kEpiGelu) {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = gelu_tanh(v[j]);
      }
      if (EPI == kEpiGatedRes || EPI == kEpiRes) {
        float g[32];
        if (EPI == kEpiGatedRes) {
          if (gate_vec) {
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              const float4 t4 = __ldg(reinterpret_cast<const float4*>(gate_row + n) + q);
              g[q * 4 + 0] = t4.x;
              g[q * 4 + 1] = t4.y;
              g[q * 4 + 2] = t4.z;
              g[q * 4 + 3] = t4.w;
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) g[j] = gate_row[n + j];
          }
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint32_t rw[4] = {rr.v[i][q].x, rr.v[i][q].y, rr.v[i][q].z, rr.v[i][q].w};
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            float2 f = unpack_bf16x2(rw[t]);
            const int j = q * 8 + t * 2;
            if (EPI == kEpiGatedRes) {
              v[j] = f.x + g[j] * v[j];
              v[j + 1] = f.y + g[j + 1] * v[j + 1];
            } else {
              v[j] = f.x + v[j];
              v[j + 1] = f.y + v[j + 1];
            }
          }
        }
      }
      uint4* cp = reinterpret_cast<uint4*>(p.C + static_cast<int64_t>(m) * p.ldc + n);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint4 o;
        o.x = pack_bf16x2(v[q * 8 + 0], v[q * 8 + 1]);
        o.y = pack_bf16x2(v[q * 8 + 2], v[q * 8 + 3]);
        o.z = pack_bf16x2(v[q * 8 + 4], v[q * 8 + 5]);
        o.w = pack_bf16x2(v[q * 8 + 6], v[q * 8 + 7]);
        cp[q] = o;
      }
    }
  }
}

template <int BN, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, EpiParams p) {
  using Cfg = GemmCfg<BN>;
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
  const int num_m = (p.M + kBM - 1) / kBM;
  const int num_n = p.N / BN;
  const int num_tiles = num_m * num_n;
  const int num_k = (p.K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int i = 0; i < ST; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 32 * kEpiWarps);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) tmem_alloc<Cfg::kTmemCols>(tmem_slot);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      int stage = 0;
      uint32_t phase = 0;
      for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
        const int m0 = (tile / num_n) * kBM;
        const int n0 = (tile % num_n) * BN;
        for (int kb = 0; kb < num_k; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, p.status, 10)) goto producer_done;
          mbar_arrive_expect_tx(&full[stage], Cfg::kABytes + Cfg::kBBytes);
          tma_load_2d(sA + stage * Cfg::kABytes, &tmA, kb * kBK, m0, &full[stage]);
          tma_load_2d(sB + stage * Cfg::kBBytes, &tmB, kb * kBK, n0, &full[stage]);
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
      constexpr uint32_t idesc = umma_idesc_bf16(kBM, BN, false);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1, abort_flag, p.status, 20)) goto mma_done;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < num_k; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, p.status, 21)) goto mma_done;
          tc_fence_after();
          const uint64_t da = umma_desc_sw128(smem_u32(sA + stage * Cfg::kABytes), 16, 1024);
          const uint64_t db = umma_desc_sw128(smem_u32(sB + stage * Cfg::kBBytes), 16, 1024);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            // advancing 16 bf16 (32 bytes) inside the swizzle atom = +2 in the >>4 address field
            umma_bf16_ss(d_tmem, da + 2 * k, db + 2 * k, idesc, (kb | k) != 0);
          }
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
    // ---------------- epilogue warps 2..9 ----------------
    // a warp may only read its TMEM lane quarter (warp % 4); the two warps of a quarter
    // split the tile's columns, so a tile drains twice as fast as with one warp per quarter
    const int quarter = warp & 3;
    const int row_in_tile = quarter * 32 + lane;
    const int col_half = (warp - 2) / 4;
    constexpr int kChunks = BN / 32;
    const int c_begin = col_half * (kChunks / 2);
    int local = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      const int m0 = (tile / num_n) * kBM;
      const int n0 = (tile % num_n) * BN;
      const int m = m0 + row_in_tile;
      const bool row_ok = m < p.M;
      ResidualRow<kChunks / 2> rr;
      prefetch_residual<kChunks / 2, EPI>(p, m, row_ok, n0, c_begin, rr);
      if (!mbar_wait(&acc_full[acc], acc_phase, abort_flag, p.status, 30)) break;
      tc_fence_after();
      const float* gate_row = nullptr;
      if (EPI == kEpiGatedRes && row_ok) {
        const int bidx = p.row_batch != nullptr ? __ldg(p.row_batch + m) : m / p.rows_per_batch;
        gate_row = p.gate + static_cast<int64_t>(bidx) * p.gate_stride;
      }
      epilogue_rows<BN, EPI, kChunks / 2>(p, tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * BN, m,
                                          row_ok, n0, gate_row, c_begin, rr);
      tc_fence_before();
      mbar_arrive(&acc_empty[acc]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (*abort_flag && threadIdx.x == 0) {
    // give copies that may still be in flight time to land before exit
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

// ---------------------------------------------------------------------------
// CTA-pair variant (cluster of two, tcgen05 cta_group::2): the pair computes a 256 x BN
// tile with M = 256 MMAs issued by the leader (cluster rank 0).  Each CTA stages its own
// 128 rows of A and its half (BN/2 rows) of B, so per FLOP a CTA pulls a third less
// operand data from L2 than with 128 x BN tiles, and each CTA's accumulator holds its own
// 128 rows.  TMA completions of both CTAs land on the leader's stage barrier (no multicast);
// the leader's commits arrive on the stage / accumulator barriers of both CTAs; the
// epilogue warps of both CTAs hand the accumulator back to the leader with a
// cluster-scope arrive.  Every wait is bounded as in the single-CTA kernel.
template <int BN>
struct Gemm2Cfg {
  static constexpr int kStages = BN == 256 ? 6 : 8;
  static constexpr int kABytes = kBM * kBK * 2;        // this CTA's 128 rows of A
  static constexpr int kBBytes = (BN / 2) * kBK * 2;   // this CTA's half of B
  static constexpr int kTmemCols = 2 * BN;
  static constexpr int kSmemBytes = kStages * (kABytes + kBBytes) + 1024 + 256;
};

template <int BN, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm2_bf16_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, EpiParams p) {
  using Cfg = Gemm2Cfg<BN>;
  constexpr int ST = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + ST * Cfg::kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + ST * Cfg::kBBytes);  // used in the leader
  uint64_t* empty = full + ST;
  uint64_t* acc_full = empty + ST;
  uint64_t* acc_empty = acc_full + 2;  // used in the leader
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // 0 = leader
  const int pair = blockIdx.x >> 1;
  const int pairs = gridDim.x >> 1;
  const int num_m = (p.M + 2 * kBM - 1) / (2 * kBM);
  const int num_n = p.N / BN;
  const int num_tiles = num_m * num_n;
  const int num_k = (p.K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int i = 0; i < ST; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 2 * kEpiWarps);  // one arrive per epilogue warp of both CTAs
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) tmem_alloc_pair<Cfg::kTmemCols>(tmem_slot);
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // the leader's barriers are initialised before the peer signals them
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer (both CTAs) ----------------
      int stage = 0;
      uint32_t phase = 0;
      for (int tile = pair; tile < num_tiles; tile += pairs) {
        const int m0 = (tile / num_n) * (2 * kBM) + static_cast<int>(rank) * kBM;
        const int n0 = (tile % num_n) * BN + static_cast<int>(rank) * (BN / 2);
        for (int kb = 0; kb < num_k; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, p.status, 40)) goto producer_done;
          const uint32_t leader_full = mapa_shared(smem_u32(&full[stage]), 0);
          if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * (Cfg::kABytes + Cfg::kBBytes));
          tma_load_2d_pair(sA + stage * Cfg::kABytes, &tmA, kb * kBK, m0, leader_full);
          tma_load_2d_pair(sB + stage * Cfg::kBBytes, &tmB, kb * kBK, n0, leader_full);
          if (++stage == ST) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    producer_done:;
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      // ---------------- MMA issuer (leader only) ----------------
      constexpr uint32_t idesc = umma_idesc_bf16(2 * kBM, BN, false);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      for (int tile = pair; tile < num_tiles; tile += pairs, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1, abort_flag, p.status, 41)) goto mma_done;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < num_k; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, p.status, 42)) goto mma_done;
          tc_fence_after();
          const uint64_t da = umma_desc_sw128(smem_u32(sA + stage * Cfg::kABytes), 16, 1024);
          const uint64_t db = umma_desc_sw128(smem_u32(sB + stage * Cfg::kBBytes), 16, 1024);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) umma_bf16_ss_pair(d_tmem, da + 2 * k, db + 2 * k, idesc, (kb | k) != 0);
          umma_commit_pair(&empty[stage]);
          if (++stage == ST) {
            stage = 0;
            phase ^= 1;
          }
        }
        umma_commit_pair(&acc_full[acc]);
      }
    mma_done:;
    }
  } else {
    // ---------------- epilogue warps 2..9 (both CTAs, own 128 rows) ----------------
    const int quarter = warp & 3;
    const int row_in_tile = quarter * 32 + lane;
    const int col_half = (warp - 2) / 4;
    constexpr int kChunks = BN / 32;
    const int c_begin = col_half * (kChunks / 2);
    int local = 0;
    for (int tile = pair; tile < num_tiles; tile += pairs, ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      const int m0 = (tile / num_n) * (2 * kBM) + static_cast<int>(rank) * kBM;
      const int n0 = (tile % num_n) * BN;
      const int m = m0 + row_in_tile;
      const bool row_ok = m < p.M;
      ResidualRow<kChunks / 2> rr;
      prefetch_residual<kChunks / 2, EPI>(p, m, row_ok, n0, c_begin, rr);
      if (!mbar_wait(&acc_full[acc], acc_phase, abort_flag, p.status, 43)) break;
      tc_fence_after();
      const float* gate_row = nullptr;
      if (EPI == kEpiGatedRes && row_ok) {
        const int bidx = p.row_batch != nullptr ? __ldg(p.row_batch + m) : m / p.rows_per_batch;
        gate_row = p.gate + static_cast<int64_t>(bidx) * p.gate_stride;
      }
      epilogue_rows<BN, EPI, kChunks / 2>(p, tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * BN, m,
                                          row_ok, n0, gate_row, c_begin, rr);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&acc_empty[acc]), 0));
    }
  }

  tc_fence_before();
  __syncthreads();
  if (*abort_flag && threadIdx.x == 0) {
    const unsigned long long t0 = globaltimer_ns();
    while (globaltimer_ns() - t0 < 1000000ull) {
    }
  }
  cluster_sync_all();  // no CTA leaves while its partner may still address its memory
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair<Cfg::kTmemCols>(tmem_base);
  }
}

template <int BN, int EPI>
void launch_pair_epi(const GemmArgs& a, cudaStream_t stream) {
  using Cfg = Gemm2Cfg<BN>;
  auto kern = gemm2_bf16_kernel<BN, EPI>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes);
  CUtensorMap tmA = make_tmap_bf16_2d(a.A, a.M, a.K, a.lda, kBM);
  CUtensorMap tmB = make_tmap_bf16_2d(a.B, a.N, a.K, a.ldb, BN / 2);
  EpiParams p;
  p.M = a.M;
  p.N = a.N;
  p.K = a.K;
  p.C = reinterpret_cast<__nv_bfloat16*>(a.C);
  p.ldc = a.ldc;
  p.bias = reinterpret_cast<const __nv_bfloat16*>(a.bias);
  p.R = reinterpret_cast<const __nv_bfloat16*>(a.R);
  p.ldr = a.ldr;
  p.gate = a.gate;
  p.gate_stride = a.gate_stride;
  p.rows_per_batch = a.rows_per_batch > 0 ? a.rows_per_batch : a.M;
  p.row_batch = a.row_batch;
  p.status = a.status;
  const int tiles = ((a.M + 2 * kBM - 1) / (2 * kBM)) * (a.N / BN);
  const int sms = a.num_sms > 0 ? a.num_sms : device_sm_count();
  const int pairs = tiles < sms / 2 ? tiles : sms / 2;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = Cfg::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, kern, tmA, tmB, p);
}

template <int BN>
void launch_pair(const GemmArgs& a, cudaStream_t stream) {
  switch (a.epilogue) {
    case kEpiNone: launch_pair_epi<BN, kEpiNone>(a, stream); break;
    case kEpiGelu: launch_pair_epi<BN, kEpiGelu>(a, stream); break;
    case kEpiGatedRes: launch_pair_epi<BN, kEpiGatedRes>(a, stream); break;
    case kEpiRes: launch_pair_epi<BN, kEpiRes>(a, stream); break;
    default: throw std::runtime_error("unknown GEMM epilogue");
  }
}

template <int BN, int EPI>
void launch_bn_epi(const GemmArgs& a, cudaStream_t stream) {
  using Cfg = GemmCfg<BN>;
  auto kern = gemm_bf16_kernel<BN, EPI>;
  // cheap host call; repeated per launch so every device gets the attribute
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes);
  CUtensorMap tmA = make_tmap_bf16_2d(a.A, a.M, a.K, a.lda, kBM);
  CUtensorMap tmB = make_tmap_bf16_2d(a.B, a.N, a.K, a.ldb, BN);
  EpiParams p;
  p.M = a.M;
  p.N = a.N;
  p.K = a.K;
  p.C = reinterpret_cast<__nv_bfloat16*>(a.C);
  p.ldc = a.ldc;
  p.bias = reinterpret_cast<const __nv_bfloat16*>(a.bias);
  p.R = reinterpret_cast<const __nv_bfloat16*>(a.R);
  p.ldr = a.ldr;
  p.gate = a.gate;
  p.gate_stride = a.gate_stride;
  p.rows_per_batch = a.rows_per_batch > 0 ? a.rows_per_batch : a.M;
  p.row_batch = a.row_batch;
  p.status = a.status;
  const int tiles = ((a.M + kBM - 1) / kBM) * (a.N / BN);
  const int sms = a.num_sms > 0 ? a.num_sms : device_sm_count();
  const int grid = tiles < sms ? tiles : sms;
  kern<<<grid, kThreads, Cfg::kSmemBytes, stream>>>(tmA, tmB, p);
}

template <int BN>
void launch_bn(const GemmArgs& a, cudaStream_t stream) {
  switch (a.epilogue) {
    case kEpiNone: launch_bn_epi<BN, kEpiNone>(a, stream); break;
    case kEpiGelu: launch_bn_epi<BN, kEpiGelu>(a, stream); break;
    case kEpiGatedRes: launch_bn_epi<BN, kEpiGatedRes>(a, stream); break;
    case kEpiRes: launch_bn_epi<BN, kEpiRes>(a, stream); break;
    default: throw std::runtime_error("unknown GEMM epilogue");
  }
}

}  // namespace

int gemm_pick_bn(int M, int N) {
  if (N % 256 == 0) {
    // prefer the wide tile unless it leaves most SMs idle on a short GEMM
    const int tiles256 = ((M + 127) / 128) * (N / 256);
    if (tiles256 >= 148 || N % 128 != 0) return 256;
    return 128;
  }
  if (N % 128 == 0) return 128;
  if (N % 64 == 0) return 64;
  return 0;
}

void launch_gemm(const GemmArgs& a, cudaStream_t stream) {
  if (a.M <= 0 || a.N <= 0 || a.K <= 0) throw std::runtime_error("gemm: empty problem");
  if (a.K % 8 != 0) throw std::runtime_error("gemm: K must be a multiple of 8");
  if ((a.epilogue == kEpiGatedRes || a.epilogue == kEpiRes) && a.R == nullptr)
    throw std::runtime_error("gemm: residual epilogue needs R");
  if (a.epilogue == kEpiGatedRes && a.gate == nullptr) throw std::runtime_error("gemm: gated epilogue needs gate");
  if ((a.ldc % 8) != 0 || (a.R && (a.ldr % 8) != 0)) throw std::runtime_error("gemm: output strides must be x8");
  static const int pair_default = [] {
    const char* e = std::getenv("DS_GEMM_PAIR");
    return e != nullptr ? (std::atoi(e) != 0 ? 1 : 0) : 1;
  }();
  const int pair = a.cta_pair >= 0 ? a.cta_pair : pair_default;
  if (pair && a.bn_override == 0) {
    // 256-row CTA-pair tiles, wide N first; by default only while the pairs still fill the
    // GPU (a forced request, cta_pair = 1, takes them whenever N allows)
    const bool forced = a.cta_pair == 1;
    const int m2 = (a.M + 2 * kBM - 1) / (2 * kBM);
    const int sms = a.num_sms > 0 ? a.num_sms : device_sm_count();
    // DS_GEMM_PAIR_MAX_BN=128 keeps pair tiles at 256 x 128 (a tuning switch; default 256)
    static const int pair_max_bn = [] {
      const char* e = std::getenv("DS_GEMM_PAIR_MAX_BN");
      return e != nullptr && std::atoi(e) == 128 ? 128 : 256;
    }();
    if (pair_max_bn == 256 && a.N % 256 == 0 && (forced || m2 * (a.N / 256) >= sms / 2)) {
      launch_pair<256>(a, stream);
      return;
    }
    if (a.N % 128 == 0 && (forced || m2 * (a.N / 128) >= sms / 2)) {
      launch_pair<128>(a, stream);
      return;
    }
  }
  const int bn = a.bn_override > 0 ? a.bn_override : gemm_pick_bn(a.M, a.N);
  if (bn == 0 || a.N % bn != 0) throw std::runtime_error("gemm: N must be a multiple of 64");
  switch (bn) {
    case 256: launch_bn<256>(a, stream); break;
    case 128: launch_bn<128>(a, stream); break;
    case 64: launch_bn<64>(a, stream); break;
    default: throw std::runtime_error("gemm: unsupported BN");
  }
}

}  // namespace ds
