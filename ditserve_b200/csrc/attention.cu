// Non-causal flash attention for sm_100a on the 5th-generation tensor cores.
//
// Layout: q, k, v, o are bf16 [tokens, heads * D] row-major views (the fused
// QKV projection output can be passed directly with its 3*H*D row stride).
// Segments are uniform (batch x seq) or ragged through cu_seqlens (token
// packing for SD3.5 continuous batching).
//
// Segments: uniform (batch x seq), ragged through cu_seqlens, or a dual-range
// table where a segment's queries and keys each come from two row ranges of the
// same buffers (MMDiT joint attention over an image block and a text block).
//
// One CTA computes two 128-row query tiles of one head of one segment (see the
// v2 comment below for the warp roles).  Softmax threads own one query row
// each (TMEM lane); O is rescaled in TMEM only when the running max grows by
// more than 2^8 (the stale max keeps P <= 256, exact in the fp32 accumulators),
// so the common iteration never touches O.  Final: O / l stored as bf16,
// optionally the natural-log LSE (ring-attention merge) or peer stores.
//
// Replaces torch SDPA (FLASH) / flash_attn_varlen_func of the reference
// (workers/ditserve/models/wan/runtime.py:442-445,
//  workers/ditserve/models/sd35_batch.py:19-117, :396-580).
#include <cstdlib>

#include "sm100.cuh"
#include "tma_host.h"
#include "kernels.h"

namespace ds {
namespace {

constexpr int kQT = 128;  // query rows per CTA
constexpr int kKT = 128;  // key rows per tile

// K/V descriptors of up to kMaxKvSources key/value sources (ring attention: the local
// chunk plus the chunks held by the ring peers, read in place over NVLink).
constexpr int kMaxKvSources = 4;
struct alignas(64) KvMaps {
  CUtensorMap k[kMaxKvSources];
  CUtensorMap v[kMaxKvSources];
};

struct AttnParams {
  int kv_sources;
  int batch, seq_q, seq_k;
  const int* cu_q;
  const int* cu_k;
  const int* seg;  // [batch][8] dual-range table (qa0 qa1 qb0 qb1 ka0 ka1 kb0 kb1) or null
  int heads, heads_kv;
  float scale_log2;  // softmax_scale * log2(e)
  float scale;
  __nv_bfloat16* o;
  int64_t o_stride;
  float* lse;
  int64_t lse_stride;
  int* status;
  int o_scatter;
  PeerGroup o_group;
  int64_t o_off;
  int o_seq_local;
  int o_head_offset;
  int64_t o_peer_stride;
  // block-sparse key tiles: query block qb (256 rows) attends to the 128-key tiles
  // blk_index[blk_offsets[qb] .. blk_offsets[qb + 1]) of its segment (null: all tiles)
  const int* blk_offsets;
  const int* blk_index;
  unsigned long long* trace;  // timeline of one CTA (kTrace instantiation only), else null
  // work list (null: one CTA per (query block, head, batch) from the grid): CTA i runs
  // work[i] = {query block | (partial slot + 1) << 16, head, batch, first key tile | end << 16};
  // a CTA with a partial slot covers a key range of its unit and leaves unnormalised O and
  // (max, sum) per row in part_o / part_ml for attention_merge
  const int4* work;
  float* part_o;    // [slots][kQBlock rows][D]
  float2* part_ml;  // [slots][kQBlock rows]
};

// Timeline instrumentation (kTrace): one CTA in the middle of the grid records SM clock
// stamps of its MMA warp and of row 0 of each softmax warpgroup for the first kTraceTiles
// key tiles: trace[j * kTraceEvents + e].  Off in every production instantiation.
constexpr int kTraceTiles = 32;
constexpr int kTraceEvents = 24;
enum TraceEvent {
  kTrVFull = 0, kTrPvA = 1, kTrSA = 2, kTrPvB = 3, kTrSB = 4,   // MMA warp
  kTrSoftBase = 5,                                               // + 5 * tile below
  kTrSFull = 0, kTrLoaded = 1, kTrMax = 2, kTrExp = 3, kTrArrive = 4,
  kTrArriveQuarter = 15,  // + quarter - 1: final P arrive of tile A rows 32, 64, 96
  kTrPWaitA = 18,         // + chunk: the MMA warp's wait for P chunk of tile A returned
  kTrEnd = 23,
};

// ---------------------------------------------------------------------------
// v2: two 128-row query tiles per CTA (A, B) and two softmax warpgroups.
//   WG0  warp 0: TMA producer (Q_A, Q_B once; K one tile ahead of V)
//        warp 1: TMEM owner + MMA issuer, order  S_A0 S_B0 | PV_A0 S_A1 PV_B0 S_B1 | ...
//   WG1  softmax of tile A (thread = row),  WG2 softmax of tile B.
// While WG1 turns S_A(j) into P_A(j) the tensor core runs S_B(j) / PV_B(j-1), and the
// other way round, so MUFU work and MMA overlap.  TMEM: S_A [0,128), S_B [128,256),
// O_A [256, 256+D), O_B [384, 384+D).  Each softmax thread loads its whole 128-column
// S row from TMEM once, takes the row max, writes bf16 P back into TMEM over the first 64
// columns of its S (the PV MMA takes P as a tensor-memory A operand, so P never touches
// shared memory) and only then rescales O (when needed): the S row and the O chunks are
// never live together and the 168-register budget of a 384-thread CTA holds without
// spills.  Shared memory holds Q_A, Q_B and two stages each of K and V.
constexpr int kAttn2Threads = 384;

// kTiles = 2 is the kernel described above.  kTiles = 1 is its short-KV form (cross-attention
// over a few hundred text keys): one 128-row Q tile and one softmax warpgroup per CTA (192
// threads: producer warp, MMA warp, softmax warps 2..5), 256 TMEM columns (S, O) and single K
// and V stages (97 KB of shared memory), so two CTAs share an SM.  With only a handful of key
// tiles per CTA, most of a CTA's life is its prologue (Q load, first QK^T) and epilogue (O
// read-out and store); a second resident CTA runs its main loop through them.
template <int D, int kTiles = 2>
struct Attn2Cfg {
  static constexpr int kAtoms = D / 64;
  static constexpr int kQBytes = kQT * D * 2;
  static constexpr int kKBytes = kKT * D * 2;
  static constexpr int kVBytes = kKT * D * 2;
  static constexpr int KS = kTiles == 2 ? 2 : 1;
  static constexpr int VS = kTiles == 2 ? 2 : 1;
  static constexpr int kSmemBytes =
      kTiles * kQBytes + KS * kKBytes + VS * kVBytes + 1024 /*align*/ + 512 /*barriers*/;
  static constexpr int kTmemCols = kTiles == 2 ? 512 : 256;
  static constexpr int kThreads = kTiles == 2 ? 384 : 192;
  static constexpr int kOBase = kTiles * 128;  // first TMEM column of O (S tiles come first)
};

__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  return (static_cast<uint64_t>(__float_as_uint(hi)) << 32) | __float_as_uint(lo);
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& lo, float& hi) {
  lo = __uint_as_float(static_cast<uint32_t>(v));
  hi = __uint_as_float(static_cast<uint32_t>(v >> 32));
}
// (a0, a1) * (b, b) + (c, c) on the packed fp32x2 datapath
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}


// kPChunks: the softmax hands P to the MMA warp in this many column chunks (one mbarrier
// phase per chunk), so the PV MMA of the first keys starts while the exponentials of the
// last keys are still being computed.
// kDiag (timeline builds only, DS_ATTN_DIAG; the output is then not attention): removes one
// ingredient of the softmax loop to see what the exponential phase is waiting on.
//   1: no P stores to tensor memory; 2: no bf16 packing; 4: no row sums; 8: a multiply instead of ex2
template <int D, int kPChunks, bool kTrace = false, int kTiles = 2, int kDiag = 0>
__global__ void __launch_bounds__(Attn2Cfg<D, kTiles>::kThreads, kTiles == 2 ? 1 : 2)
    attention2_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ KvMaps kv,
                      AttnParams p) {
  using Cfg = Attn2Cfg<D, kTiles>;
  constexpr int KS = Cfg::KS;
  constexpr int VS = Cfg::VS;
  constexpr int kQBlock = kTiles * kQT;  // query rows per CTA
  int qblk = blockIdx.x, h = blockIdx.y, b = blockIdx.z, slot = -1, kv_first = 0, kv_end = -1;
  if (p.work != nullptr) {
    const int4 wd = p.work[blockIdx.x];
    qblk = wd.x & 0xffff;
    slot = (wd.x >> 16) - 1;
    h = wd.y;
    b = wd.z;
    kv_first = wd.w & 0xffff;
    kv_end = wd.w >> 16;
  }
  // segment = query rows [qa0,qa1) u [qb0,qb1) attending to keys [ka0,ka1) u [kb0,kb1)
  int qa0, qa1, qb0, qb1, ka0, ka1, kb0, kb1;
  if (p.seg != nullptr) {
    const int* sg = p.seg + 8 * b;
    qa0 = sg[0]; qa1 = sg[1]; qb0 = sg[2]; qb1 = sg[3];
    ka0 = sg[4]; ka1 = sg[5]; kb0 = sg[6]; kb1 = sg[7];
  } else if (p.cu_q != nullptr) {
    qa0 = p.cu_q[b]; qa1 = p.cu_q[b + 1];
    ka0 = p.cu_k[b]; ka1 = p.cu_k[b + 1];
    qb0 = qb1 = kb0 = kb1 = 0;
  } else {
    qa0 = b * p.seq_q; qa1 = qa0 + p.seq_q;
    ka0 = b * p.seq_k; ka1 = ka0 + p.seq_k;
    qb0 = qb1 = kb0 = kb1 = 0;
  }
  const int nqa = (qa1 - qa0 + kQBlock - 1) / kQBlock;
  const int nqb = (qb1 - qb0 + kQBlock - 1) / kQBlock;
  int q0, q_end;
  if (qblk < nqa) {
    q0 = qa0 + qblk * kQBlock;
    q_end = qa1;
  } else if (qblk < nqa + nqb) {
    q0 = qb0 + (qblk - nqa) * kQBlock;
    q_end = qb1;
  } else {
    return;
  }
  const int nka = (ka1 - ka0 + kKT - 1) / kKT;
  const int* blk = nullptr;  // block-sparse: this query block's list of key tiles
  int per_source = nka + (kb1 - kb0 + kKT - 1) / kKT;
  if (p.blk_offsets != nullptr) {
    const int o0 = p.blk_offsets[qblk];
    blk = p.blk_index + o0;
    per_source = p.blk_offsets[qblk + 1] - o0;
  }
  int kv_base = 0;  // work-list CTAs start at their first key tile (one source, one range)
  if (p.work != nullptr) {
    kv_base = kv_first;
    per_source = kv_end - kv_first;
  }
  const int n_tiles = per_source * p.kv_sources;
  if (n_tiles <= 0) return;  // uniform across the CTA
  // tile j reads source j / per_source; within a source the segment's key ranges repeat
  auto ktile_row = [&](int j) {
    const int jj = j % per_source + kv_base;
    if (blk != nullptr) return ka0 + blk[jj] * kKT;
    return jj < nka ? ka0 + jj * kKT : kb0 + (jj - nka) * kKT;
  };
  auto ktile_valid = [&](int j) {
    const int jj = j % per_source + kv_base;
    if (blk != nullptr) return ka1 - (ka0 + blk[jj] * kKT);
    return jj < nka ? ka1 - (ka0 + jj * kKT) : kb1 - (kb0 + (jj - nka) * kKT);
  };
  const int hk = h / (p.heads / p.heads_kv);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                                   // [2][kQBytes]
  uint8_t* sK = sQ + kTiles * Cfg::kQBytes;             // [KS][kKBytes]
  uint8_t* sV = sK + KS * Cfg::kKBytes;                 // [VS][kVBytes]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + VS * Cfg::kVBytes);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* k_empty = k_full + KS;
  uint64_t* v_full = k_empty + KS;
  uint64_t* v_empty = v_full + VS;
  uint64_t* s_full = v_empty + VS;  // [2] per tile
  uint64_t* p_full = s_full + kTiles;    // [kTiles][kPChunks]
  uint64_t* pv_done = p_full + kTiles * kPChunks;  // [kTiles]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(pv_done + kTiles);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int wg = warp >> 2;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < KS; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < VS; ++i) {
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < kTiles; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&pv_done[i], 1);
    }
    for (int i = 0; i < kTiles * kPChunks; ++i) mbar_init(&p_full[i], 128);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc<Cfg::kTmemCols>(tmem_slot);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const bool tracing = kTrace && p.trace != nullptr && qblk == static_cast<int>(gridDim.x / 2) && blockIdx.y == 0 &&
                       blockIdx.z == 0;
  auto rec = [&](int j, int e) {
    if (kTrace && tracing && j < kTraceTiles) p.trace[j * kTraceEvents + e] = clock64();
  };

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer: K runs one tile ahead of V ----------------
      tma_prefetch_desc(&tmQ);
      for (int src = 0; src < p.kv_sources; ++src) {
        tma_prefetch_desc(&kv.k[src]);
        tma_prefetch_desc(&kv.v[src]);
      }
      mbar_arrive_expect_tx(q_full, kTiles * Cfg::kQBytes);
#pragma unroll
      for (int t = 0; t < kTiles; ++t)
#pragma unroll
        for (int a = 0; a < Cfg::kAtoms; ++a)
          tma_load_2d(sQ + t * Cfg::kQBytes + a * (kQT * 128), &tmQ, h * D + a * 64, q0 + t * kQT, q_full);
      auto load_k = [&](int j) -> bool {
        const int st = j % KS;
        if (!mbar_wait(&k_empty[st], ((j / KS) & 1) ^ 1, abort_flag, p.status, 210)) return false;
        mbar_arrive_expect_tx(&k_full[st], Cfg::kKBytes);
#pragma unroll
        for (int a = 0; a < Cfg::kAtoms; ++a)
          tma_load_2d(sK + st * Cfg::kKBytes + a * (kKT * 128), &kv.k[j / per_source], hk * D + a * 64, ktile_row(j),
                      &k_full[st]);
        return true;
      };
      bool ok = load_k(0);
      for (int j = 0; ok && j < n_tiles; ++j) {
        if (j + 1 < n_tiles && !load_k(j + 1)) break;
        const int st = j % VS;
        if (!mbar_wait(&v_empty[st], ((j / VS) & 1) ^ 1, abort_flag, p.status, 211)) break;
        mbar_arrive_expect_tx(&v_full[st], Cfg::kVBytes);
#pragma unroll
        for (int a = 0; a < Cfg::kAtoms; ++a)
          tma_load_2d(sV + st * Cfg::kVBytes + a * (kKT * 128), &kv.v[j / per_source], hk * D + a * 64, ktile_row(j),
                      &v_full[st]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      constexpr uint32_t idesc_s = umma_idesc_bf16(kQT, kKT, false);
      constexpr uint32_t idesc_o = umma_idesc_bf16(kQT, D, true);
      auto issue_s = [&](int t, int j) {
        const int st = j % KS;
        const uint32_t d = tmem_base + t * kKT;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * (kQT * 128) + (kk & 3) * 32;
          const uint64_t da = umma_desc_sw128(smem_u32(sQ + t * Cfg::kQBytes) + off, 16, 1024);
          const uint64_t db = umma_desc_sw128(smem_u32(sK + st * Cfg::kKBytes) + off, 16, 1024);
          umma_bf16_ss(d, da, db, idesc_s, kk != 0);
        }
        umma_commit(&s_full[t]);
      };
      auto issue_pv = [&](int t, int j) -> bool {
        const uint32_t d = tmem_base + Cfg::kOBase + t * 128;
        const uint32_t p_tmem = tmem_base + t * kKT;  // bf16 P packed over the first 64 S columns
        const uint32_t v_base = smem_u32(sV + (j % VS) * Cfg::kVBytes);
        constexpr int kPerChunk = kKT / 16 / kPChunks;  // K=16 MMAs per P chunk
#pragma unroll
        for (int c = 0; c < kPChunks; ++c) {
          if (!mbar_wait(&p_full[t * kPChunks + c], j & 1, abort_flag, p.status, 222 + t)) return false;
          if (t == 0 && c < 2) rec(j, kTrPWaitA + c);
          tc_fence_after();
#pragma unroll
          for (int i = 0; i < kPerChunk; ++i) {
            const int kk = c * kPerChunk + i;
            const uint64_t db = umma_desc_sw128(v_base + kk * (16 * 128), kKT * 128, 1024);
            umma_bf16_ts(d, p_tmem + kk * 8, db, idesc_o, (j | kk) != 0);
          }
        }
        umma_commit(&pv_done[t]);
        return true;
      };
      bool ok = mbar_wait(q_full, 0, abort_flag, p.status, 220) &&
                mbar_wait(&k_full[0], 0, abort_flag, p.status, 221);
      if (ok) {
        tc_fence_after();
        issue_s(0, 0);
        if (kTiles == 2) issue_s(1, 0);
        umma_commit(&k_empty[0]);
      }
      for (int j = 0; ok && kTiles == 1 && j < n_tiles; ++j) {
        // one Q tile: PV(j), then S(j+1) into the columns P(j) occupied
        if (!mbar_wait(&v_full[j % VS], (j / VS) & 1, abort_flag, p.status, 224)) break;
        tc_fence_after();
        if (!issue_pv(0, j)) break;
        umma_commit(&v_empty[j % VS]);
        if (j + 1 < n_tiles) {
          const int st = (j + 1) % KS;
          if (!mbar_wait(&k_full[st], ((j + 1) / KS) & 1, abort_flag, p.status, 225)) break;
          tc_fence_after();
          issue_s(0, j + 1);
          umma_commit(&k_empty[st]);
        }
      }
      for (int j = 0; ok && kTiles == 2 && j < n_tiles; ++j) {
        if (!mbar_wait(&v_full[j % VS], (j / VS) & 1, abort_flag, p.status, 224)) break;
        rec(j, kTrVFull);
        tc_fence_after();
        if (!issue_pv(0, j)) break;
        rec(j, kTrPvA);
        const bool more = j + 1 < n_tiles;
        if (more) {
          const int st = (j + 1) % KS;
          if (!mbar_wait(&k_full[st], ((j + 1) / KS) & 1, abort_flag, p.status, 225)) break;
          tc_fence_after();
          issue_s(0, j + 1);
          rec(j, kTrSA);
        }
        if (!issue_pv(1, j)) break;
        rec(j, kTrPvB);
        umma_commit(&v_empty[j % VS]);
        if (more) {
          issue_s(1, j + 1);
          umma_commit(&k_empty[(j + 1) % KS]);
          rec(j, kTrSB);
        }
      }
    }
  } else if (kTiles == 2 ? wg >= 1 : warp >= 2) {
    // ---------------- softmax warpgroups (tile t = wg - 1; warps 2..5 when kTiles = 1) ----------------
    const int t = kTiles == 2 ? wg - 1 : 0;
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t s_col = tmem_base + lane_addr + t * kKT;
    const uint32_t o_col = tmem_base + lane_addr + Cfg::kOBase + t * 128;
    const float sl2 = p.scale_log2;
    const uint64_t sl2x2 = f2_pack(sl2, sl2);
    float m_run = -INFINITY;
    float l_run = 0.f;
    bool ok = true;
    const bool trace_row = row == 0;
    auto srec = [&](int j, int e) {
      if (kTrace && trace_row) rec(j, kTrSoftBase + 5 * t + e);
      if (kTrace && e == kTrArrive && t == 0 && lane == 0 && quarter > 0) rec(j, kTrArriveQuarter + quarter - 1);
    };
    for (int j = 0; j < n_tiles; ++j) {
      if (!mbar_wait(&s_full[t], j & 1, abort_flag, p.status, 230 + t)) {
        ok = false;
        break;
      }
      srec(j, kTrSFull);
      tc_fence_after();
      const int valid = ktile_valid(j);  // columns >= valid are outside the segment
      const bool masked = valid < kKT;
      // one pass over TMEM: the thread's whole 128-column S row into registers
      uint32_t s[kKT];
#pragma unroll
      for (int c = 0; c < kKT / 32; ++c)
        tmem_ld32(s_col + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&s[c * 32]));
      tmem_wait_ld();
      srec(j, kTrLoaded);
      float mx = -INFINITY;
      if (masked) {
#pragma unroll
        for (int c = 0; c < kKT; ++c)
          if (c < valid) mx = fmaxf(mx, __uint_as_float(s[c]));
      } else {
        float mc[8];  // eight independent chains keep the dependent max sequence short
#pragma unroll
        for (int i = 0; i < 8; ++i) mc[i] = __uint_as_float(s[i]);
#pragma unroll
        for (int c = 8; c < kKT; c += 8)
#pragma unroll
          for (int i = 0; i < 8; ++i) mc[i] = fmaxf(mc[i], __uint_as_float(s[c + i]));
        mx = fmaxf(fmaxf(fmaxf(mc[0], mc[1]), fmaxf(mc[2], mc[3])), fmaxf(fmaxf(mc[4], mc[5]), fmaxf(mc[6], mc[7])));
      }
      const float m_new = fmaxf(m_run, mx);
      srec(j, kTrMax);
      const bool need = (m_new - m_run) * sl2 > 8.0f;  // always true on the first tile
      float alpha = 1.f;
      if (need) {
        alpha = ex2_approx((m_run - m_new) * sl2);
        m_run = m_new;
      }
      if (j > 0) {
        // PV(j-1) has completed (the commit behind S(j) covers it); wait formally so the
        // P overwrite and the O rescale below are ordered after it
        if (!mbar_wait(&pv_done[t], (j - 1) & 1, abort_flag, p.status, 232 + t)) {
          ok = false;
          break;
        }
        tc_fence_after();
      }
      l_run *= alpha;
      const float neg = -m_run * sl2;
      const uint64_t negx2 = f2_pack(neg, neg);
      float ls[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};  // per-column-slot partial row sums
      int signalled = 0;  // P chunks (of 8 columns) already handed to the MMA warp
      // exponentials, row sum, bf16 P into tensor memory; masked tiles
      // (a segment's last) take their own loop so the common tile carries no column tests.
      // (Moving a quarter or half of the exponentials to an FMA-pipe polynomial measured
      // 6-13 % slower than all-MUFU here, so every exponential uses ex2.approx.)
      // P goes back into TMEM over the first 64 columns of this tile's S (the S row is in
      // registers already): 8 packed columns per store, the PV MMA reads it as its A operand
      uint32_t pk8[8];
      auto p_chunk = [&](int ch, float (&e8)[8]) {
        const int q = (ch & 1) * 4;
        if (kDiag & 2) {
          pk8[q + 0] = __float_as_uint(e8[0]) ^ __float_as_uint(e8[1]);
          pk8[q + 1] = __float_as_uint(e8[2]) ^ __float_as_uint(e8[3]);
          pk8[q + 2] = __float_as_uint(e8[4]) ^ __float_as_uint(e8[5]);
          pk8[q + 3] = __float_as_uint(e8[6]) ^ __float_as_uint(e8[7]);
        } else {
          pk8[q + 0] = pack_bf16x2(e8[0], e8[1]);
          pk8[q + 1] = pack_bf16x2(e8[2], e8[3]);
          pk8[q + 2] = pack_bf16x2(e8[4], e8[5]);
          pk8[q + 3] = pack_bf16x2(e8[6], e8[7]);
        }
        if (kDiag & 1) {
          if (ch == kKT / 8 - 1) tmem_st8(s_col, pk8);  // keep one store so the values stay live
        } else if (ch & 1) {
          tmem_st8(s_col + (ch >> 1) * 8, pk8);
        }
      };
      if (masked) {
#pragma unroll
        for (int ch = 0; ch < kKT / 8; ++ch) {
          float e8[8];
#pragma unroll
          for (int e = 0; e < 8; e += 2) {
            const int c = ch * 8 + e;
            const uint64_t x2 = f2_fma(f2_pack(__uint_as_float(s[c]), __uint_as_float(s[c + 1])), sl2x2, negx2);
            float x0, x1;
            f2_unpack(x2, x0, x1);
            if (c >= valid) x0 = -INFINITY;
            if (c + 1 >= valid) x1 = -INFINITY;
            e8[e] = ex2_approx(x0);
            e8[e + 1] = ex2_approx(x1);
            ls[e] += e8[e];
            ls[e + 1] += e8[e + 1];
          }
          p_chunk(ch, e8);
        }
      } else {
        // with no O rescale pending in this warp (the common case), each finished P chunk is
        // handed to the MMA warp at once; otherwise all chunks go after the rescale below
        const bool early = kPChunks > 1 && !(j > 0 && __any_sync(0xffffffffu, need));
        constexpr int kChunkCh = kKT / 8 / kPChunks;  // 8-column steps per P chunk
#pragma unroll
        for (int ch = 0; ch < kKT / 8; ++ch) {
          float e8[8];
#pragma unroll
          for (int e = 0; e < 8; e += 2) {
            const int c = ch * 8 + e;
            const uint64_t x2 = f2_fma(f2_pack(__uint_as_float(s[c]), __uint_as_float(s[c + 1])), sl2x2, negx2);
            float x0, x1;
            f2_unpack(x2, x0, x1);
            if (kDiag & 8) {
              e8[e] = x0 * 0.5f;
              e8[e + 1] = x1 * 0.5f;
            } else {
              e8[e] = ex2_approx(x0);
              e8[e + 1] = ex2_approx(x1);
            }
            if (!(kDiag & 4)) {
              ls[e] += e8[e];
              ls[e + 1] += e8[e + 1];
            }
          }
          if (kDiag & 4) ls[0] += e8[7];
          p_chunk(ch, e8);
          if (kPChunks > 1 && early && ((ch + 1) % kChunkCh) == 0) {
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(&p_full[t * kPChunks + (ch + 1) / kChunkCh - 1]);
            signalled = ch + 1;
          }
        }
      }
      l_run += ((ls[0] + ls[1]) + (ls[2] + ls[3])) + ((ls[4] + ls[5]) + (ls[6] + ls[7]));
      srec(j, kTrExp);
      // O rescale after the exponentials: the S row is dead by now, so the O chunks do not
      // add to the peak register use; PV(j) only starts after p_full below
      if (j > 0 && __any_sync(0xffffffffu, need)) {
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o[32];
          tmem_ld32(o_col + c * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
          tmem_st32(o_col + c * 32, o);
        }
        tmem_wait_st();
      }
      tmem_wait_st();
      tc_fence_before();
      for (int c = signalled / (kKT / 8 / kPChunks); c < kPChunks; ++c) mbar_arrive(&p_full[t * kPChunks + c]);
      srec(j, kTrArrive);
    }
    if (ok) ok = mbar_wait(&pv_done[t], (n_tiles - 1) & 1, abort_flag, p.status, 234 + t);
    if (ok && slot >= 0) {
      // partial unit: unnormalised O and (max, sum) of this key range, merged by attention_merge
      tc_fence_after();
      const int64_t prow = static_cast<int64_t>(slot) * kQBlock + t * kQT + row;
      float4* dst = reinterpret_cast<float4*>(p.part_o + prow * D);
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        tmem_ld32(o_col + c * 32, o);
        tmem_wait_ld();
#pragma unroll
        for (int q = 0; q < 8; ++q)
          dst[c * 8 + q] = make_float4(__uint_as_float(o[q * 4]), __uint_as_float(o[q * 4 + 1]),
                                       __uint_as_float(o[q * 4 + 2]), __uint_as_float(o[q * 4 + 3]));
      }
      p.part_ml[prow] = make_float2(m_run, l_run);
      ok = false;  // the bf16 epilogue below is the merge kernel's job
    }
    if (ok) {
      tc_fence_after();
      const int qabs = q0 + t * kQT + row;  // absolute row of q / o
      const bool row_ok = qabs < q_end;
      const float inv_l = 1.0f / l_run;
      __nv_bfloat16* orow;
      if (p.o_scatter) {
        // Ulysses head->sequence all-to-all: the row goes straight to the token's owner
        const int qrow = qabs - qa0;
        const int owner = qrow / p.o_seq_local;
        const int local = qrow - owner * p.o_seq_local;
        __nv_bfloat16* base = reinterpret_cast<__nv_bfloat16*>(
            reinterpret_cast<uint8_t*>(p.o_group.base[owner < p.o_group.size ? owner : 0]) + p.o_off);
        orow = base + (static_cast<int64_t>(b) * p.o_seq_local + local) * p.o_peer_stride + (p.o_head_offset + h) * D;
      } else {
        orow = p.o + static_cast<int64_t>(qabs) * p.o_stride + h * D;
      }
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        tmem_ld32(o_col + c * 32, o);
        tmem_wait_ld();
        if (row_ok) {
          uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 w;
            w.x = pack_bf16x2(__uint_as_float(o[q * 8 + 0]) * inv_l, __uint_as_float(o[q * 8 + 1]) * inv_l);
            w.y = pack_bf16x2(__uint_as_float(o[q * 8 + 2]) * inv_l, __uint_as_float(o[q * 8 + 3]) * inv_l);
            w.z = pack_bf16x2(__uint_as_float(o[q * 8 + 4]) * inv_l, __uint_as_float(o[q * 8 + 5]) * inv_l);
            w.w = pack_bf16x2(__uint_as_float(o[q * 8 + 6]) * inv_l, __uint_as_float(o[q * 8 + 7]) * inv_l);
            dst[q] = w;
          }
        }
      }
      if (row_ok && p.lse != nullptr)
        p.lse[static_cast<int64_t>(h) * p.lse_stride + qabs] = m_run * p.scale + logf(l_run);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (kTrace && tracing && threadIdx.x == 0) p.trace[kTrEnd] = clock64();
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

// Combines the key-range partials of split units: one warp per (unit, query row).  With
// part i = (m_i, l_i, O_i) over its key range, M = max m_i, w_i = 2^((m_i - M) * scale_log2):
// O = sum w_i O_i / sum w_i l_i and LSE = M * scale + ln(sum w_i l_i).  The row is written
// where the attention epilogue would have written it (locally or into its owner's buffer).
struct MergeParams {
  const int4* units;  // {query block, head, batch, first slot | parts << 16}
  int num_units;
  const float* part_o;
  const float2* part_ml;
  int seq_q;
  float scale_log2, scale;
  __nv_bfloat16* o;
  int64_t o_stride;
  float* lse;
  int64_t lse_stride;
  int o_scatter;
  PeerGroup o_group;
  int64_t o_off;
  int o_seq_local;
  int o_head_offset;
  int64_t o_peer_stride;
};

template <int D, int kQBlock>
__global__ void __launch_bounds__(256) attention_merge_kernel(MergeParams p) {
  constexpr int kPer = D / 32;  // columns per lane
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int unit = gw / kQBlock;
  const int r = gw - unit * kQBlock;
  if (unit >= p.num_units) return;
  const int4 u = p.units[unit];
  const int q = u.x * kQBlock + r;
  if (q >= p.seq_q) return;
  const int h = u.y, b = u.z, slot0 = u.w & 0xffff, parts = u.w >> 16;
  float mmax = -INFINITY;
  for (int i = 0; i < parts; ++i) mmax = fmaxf(mmax, p.part_ml[static_cast<int64_t>(slot0 + i) * kQBlock + r].x);
  float acc[kPer];
#pragma unroll
  for (int e = 0; e < kPer; ++e) acc[e] = 0.f;
  float lsum = 0.f;
  for (int i = 0; i < parts; ++i) {
    const int64_t prow = static_cast<int64_t>(slot0 + i) * kQBlock + r;
    const float2 ml = p.part_ml[prow];
    const float w = ex2_approx((ml.x - mmax) * p.scale_log2);
    lsum += w * ml.y;
    const float* src = p.part_o + prow * D + lane * kPer;
#pragma unroll
    for (int e = 0; e < kPer; ++e) acc[e] += w * src[e];
  }
  const float inv = 1.0f / lsum;
  __nv_bfloat16* orow;
  if (p.o_scatter) {
    const int owner = q / p.o_seq_local;
    const int local = q - owner * p.o_seq_local;
    __nv_bfloat16* base = reinterpret_cast<__nv_bfloat16*>(
        reinterpret_cast<uint8_t*>(p.o_group.base[owner < p.o_group.size ? owner : 0]) + p.o_off);
    orow = base + (static_cast<int64_t>(b) * p.o_seq_local + local) * p.o_peer_stride + (p.o_head_offset + h) * D;
  } else {
    orow = p.o + (static_cast<int64_t>(b) * p.seq_q + q) * p.o_stride + h * D;
  }
  if (kPer == 4) {
    uint2 v;
    v.x = pack_bf16x2(acc[0] * inv, acc[1] * inv);
    v.y = pack_bf16x2(acc[2 % kPer] * inv, acc[3 % kPer] * inv);
    *reinterpret_cast<uint2*>(orow + lane * kPer) = v;
  } else {
    *reinterpret_cast<uint32_t*>(orow + lane * kPer) = pack_bf16x2(acc[0] * inv, acc[1 % kPer] * inv);
  }
  if (lane == 0 && p.lse != nullptr)
    p.lse[static_cast<int64_t>(h) * p.lse_stride + static_cast<int64_t>(b) * p.seq_q + q] = mmax * p.scale + logf(lsum);
}

template <int D>
void launch_d(const AttnArgs& a, cudaStream_t stream) {
  CUtensorMap tq = make_tmap_bf16_2d(a.q, a.total_q, static_cast<uint64_t>(a.heads) * D, a.q_row_stride, kQT);
  if (a.kv_sources < 1 || a.kv_sources > kMaxKvSources) throw std::runtime_error("attention: 1..4 KV sources");
  KvMaps kv;
  for (int src = 0; src < a.kv_sources; ++src) {
    const void* kp = src == 0 ? a.k : a.k_extra[src - 1];
    const void* vp = src == 0 ? a.v : a.v_extra[src - 1];
    if (kp == nullptr || vp == nullptr) throw std::runtime_error("attention: missing KV source pointer");
    kv.k[src] = make_tmap_bf16_2d(kp, a.total_k, static_cast<uint64_t>(a.heads_kv) * D, a.k_row_stride, kKT);
    kv.v[src] = make_tmap_bf16_2d(vp, a.total_k, static_cast<uint64_t>(a.heads_kv) * D, a.v_row_stride, kKT);
  }
  AttnParams p;
  p.kv_sources = a.kv_sources;
  p.batch = a.batch;
  p.seq_q = a.seq_q;
  p.seq_k = a.seq_k;
  p.cu_q = a.cu_seqlens_q;
  p.cu_k = a.cu_seqlens_k;
  p.seg = a.seg_table;
  p.heads = a.heads;
  p.heads_kv = a.heads_kv;
  p.scale = a.softmax_scale;
  p.scale_log2 = a.softmax_scale * 1.4426950408889634f;
  p.o = reinterpret_cast<__nv_bfloat16*>(a.o);
  p.o_stride = a.o_row_stride;
  p.lse = a.lse;
  p.lse_stride = a.lse_stride;
  p.status = a.status;
  p.o_scatter = a.o_scatter;
  p.o_group = a.o_group;
  p.o_off = a.o_off;
  p.o_seq_local = a.o_seq_local;
  p.o_head_offset = a.o_head_offset;
  p.o_peer_stride = a.o_peer_stride;
  p.blk_offsets = a.blk_offsets;
  p.blk_index = a.blk_index;
  p.work = a.work;
  p.part_o = a.part_o;
  p.part_ml = reinterpret_cast<float2*>(a.part_ml);
  if (a.work != nullptr && (a.seg_table != nullptr || a.cu_seqlens_q != nullptr || a.blk_offsets != nullptr ||
                            a.kv_sources != 1 || a.trace != nullptr))
    throw std::runtime_error("attention: a work list needs uniform batches, one KV source, no sparse table");
  if (a.blk_offsets != nullptr && (a.seg_table != nullptr || a.kv_sources != 1))
    throw std::runtime_error("attention: block-sparse key tiles need one KV source and no dual-range table");
  // grid.x: 256-row query blocks of the longest segment (both ranges in dual-range mode)
  const int max_q = (a.cu_seqlens_q || a.seg_table) ? a.max_seq_q : a.seq_q;
  const int blocks = a.seg_table ? a.max_q_blocks : (max_q + 2 * kQT - 1) / (2 * kQT);
  // P hand-off granularity (DS_ATTN_PCHUNKS = 1, 2 or 4; default 2)
  static const int pchunks = [] {
    const char* e = std::getenv("DS_ATTN_PCHUNKS");
    const int v = e != nullptr ? std::atoi(e) : 2;
    return v == 1 || v == 4 ? v : 2;
  }();
  p.trace = a.trace;
  // short key ranges (cross-attention): one Q tile per CTA, two CTAs per SM.  Uniform batches
  // only (the 256-row block numbering of the dual-range and block-sparse tables stays as is);
  // DS_ATTN_SHORT_KV sets the largest key count that takes this form (default 1024, 0: never)
  static const int short_kv = [] {
    const char* e = std::getenv("DS_ATTN_SHORT_KV");
    return e != nullptr ? std::atoi(e) : 1024;
  }();
  const bool uniform = a.cu_seqlens_q == nullptr && a.seg_table == nullptr && a.blk_offsets == nullptr;
  if (uniform && a.trace == nullptr && a.work == nullptr && static_cast<int64_t>(a.seq_k) * a.kv_sources <= short_kv) {
    using C1 = Attn2Cfg<D, 1>;
    auto kern1 = attention2_kernel<D, 2, false, 1>;
    cudaFuncSetAttribute(kern1, cudaFuncAttributeMaxDynamicSharedMemorySize, C1::kSmemBytes);
    dim3 grid1((a.seq_q + kQT - 1) / kQT, a.heads, a.batch);
    kern1<<<grid1, C1::kThreads, C1::kSmemBytes, stream>>>(tq, kv, p);
    return;
  }
  auto kern = a.trace != nullptr ? attention2_kernel<D, 2, true>
              : pchunks == 1     ? attention2_kernel<D, 1>
              : pchunks == 4     ? attention2_kernel<D, 4>
                                 : attention2_kernel<D, 2>;
  if (a.trace != nullptr && D == 128) {
    static const int diag = [] {
      const char* e = std::getenv("DS_ATTN_DIAG");
      return e != nullptr ? std::atoi(e) : 0;
    }();
    switch (diag) {
      case 1: kern = attention2_kernel<D, 2, true, 2, 1>; break;
      case 2: kern = attention2_kernel<D, 2, true, 2, 2>; break;
      case 4: kern = attention2_kernel<D, 2, true, 2, 4>; break;
      case 8: kern = attention2_kernel<D, 2, true, 2, 8>; break;
      case 15: kern = attention2_kernel<D, 2, true, 2, 15>; break;
      default: break;
    }
  }
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Attn2Cfg<D>::kSmemBytes);
  if (a.work != nullptr) {
    // work list: whole units first, then the key-range parts of the tail units; the merge
    // kernel runs after them on the same stream
    kern<<<a.num_work, kAttn2Threads, Attn2Cfg<D>::kSmemBytes, stream>>>(tq, kv, p);
    if (a.num_merge_units > 0) {
      MergeParams mp;
      mp.units = a.merge_units;
      mp.num_units = a.num_merge_units;
      mp.part_o = a.part_o;
      mp.part_ml = reinterpret_cast<const float2*>(a.part_ml);
      mp.seq_q = a.seq_q;
      mp.scale_log2 = p.scale_log2;
      mp.scale = p.scale;
      mp.o = p.o;
      mp.o_stride = p.o_stride;
      mp.lse = p.lse;
      mp.lse_stride = p.lse_stride;
      mp.o_scatter = p.o_scatter;
      mp.o_group = p.o_group;
      mp.o_off = p.o_off;
      mp.o_seq_local = p.o_seq_local;
      mp.o_head_offset = p.o_head_offset;
      mp.o_peer_stride = p.o_peer_stride;
      const int warps = a.num_merge_units * 2 * kQT;
      attention_merge_kernel<D, 2 * kQT><<<(warps + 7) / 8, 256, 0, stream>>>(mp);
    }
    return;
  }
  dim3 grid(blocks, a.heads, a.batch);
  kern<<<grid, kAttn2Threads, Attn2Cfg<D>::kSmemBytes, stream>>>(tq, kv, p);
}

}  // namespace

void launch_attention(const AttnArgs& a, cudaStream_t stream) {
  if (a.heads <= 0 || a.heads_kv <= 0 || a.heads % a.heads_kv != 0) throw std::runtime_error("attention: bad heads");
  if (a.q_row_stride % 8 || a.k_row_stride % 8 || a.v_row_stride % 8 || a.o_row_stride % 8)
    throw std::runtime_error("attention: row strides must be multiples of 8 elements");
  if ((a.cu_seqlens_q == nullptr) != (a.cu_seqlens_k == nullptr))
    throw std::runtime_error("attention: give both cu_seqlens or neither");
  if (a.cu_seqlens_q != nullptr && a.max_seq_q <= 0) throw std::runtime_error("attention: max_seq_q required");
  if (a.seg_table != nullptr && a.max_q_blocks <= 0) throw std::runtime_error("attention: max_q_blocks required");
  switch (a.head_dim) {
    case 128: launch_d<128>(a, stream); break;
    case 64: launch_d<64>(a, stream); break;
    default: throw std::runtime_error("attention: head_dim must be 64 or 128");
  }
}

}  // namespace ds
