// FlashAttention forward for B200 (sm_100a): fp16 Q/K/V in [B, H, N, 64]
// layout, fp32 accumulation, fp16 output, optional top-left causal mask.
//
// It replaces the sm_80-style production kernel of the reference
// (csrc/tensorcore_attention.cu:2019-2727, launched from :2969-3123) with a
// warp-specialized, persistent tcgen05 design:
//
//   warp 8      TMA producer: Q tiles of the current work item, then K_j/V_j
//               tiles through a ring of swizzled shared-memory slots.
//   warp 10     MMA issuer (one elected lane) for S_t = Q_t K_j^T (SS form).
//   warp 11     MMA issuer for O_t += P_t V_j (P read straight from tensor
//               memory, TS form).  Issuing tcgen05.mma slows the softmax
//               warps of the same SM sub-partition, so the two issue streams
//               sit on different sub-partitions.
//   warp 9      owns the tensor-memory allocation, otherwise idle.
//   warps 0-3   softmax for query tile 0 of the work item, one thread per row.
//   warps 4-7   softmax for query tile 1 (ping-pong partner of tile 0).
//
// A work item is one (batch*head, query-pair) unit: 256 query rows as two
// 128-row tiles (one tile per item for short problems; with a key-range split
// for few long heads, also one split of the keys).  Tensor memory (512
// columns) holds, per tile t,
//   S_t  128 x 128 fp32   (columns   0 / 128)
//   O_t  128 x  64 fp32   (columns 256 / 320)
//   P_t  128 x 128 fp16   (columns 384 / 448, two halves per column)
// so S_t(j+1) can be computed while the softmax warps are still turning
// S_t(j) into P_t(j).  Each softmax warp writes its 32 rows of the normalised
// output with its own TMA store.  The two softmax warpgroups take turns on
// the MUFU (16 ex2/clk/SM, the unit that bounds attention at head dimension
// 64): one tile's exponentials overlap the other tile's S load, row max and
// P store.
//
// Online softmax follows the reference's tile update
// (csrc/tensorcore_attention.cu:448-671): running row max m, running sum l,
// p = exp(s*scale - m), O rescaled by exp(m_old - m_new).  The max used for
// the exponent is only moved when the row max grows by more than 2^8 in the
// exponent, which keeps every p <= 256 (well inside fp16 range) and skips
// most O rescales; the final O / l is unchanged because both use the same max.
//
// Every wait is bounded in time.  A wait that runs out sets a bit in a device
// status word, sets a shared abort flag that releases the other roles, and the
// block drains its in-flight copies and frees tensor memory before returning.

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <algorithm>
#include <atomic>
#include <map>
#include <memory>
#include <mutex>
#include <utility>

#include "sm100_ptx.cuh"
#include "fa_sm100.h"

#ifndef FA_TRACE
#define FA_TRACE 0
#endif
#ifndef FA_POLY_PAIRS
#define FA_POLY_PAIRS 0  // of every 8 exponent pairs, this many use the FMA-pipe polynomial
                         // (0 measured fastest in this kernel on a B200)
#endif
// Roles of the third warpgroup (warps 8-11): the producer and the MMA issuers
// must be different warps of that group, except that one warp may issue both
// kinds of MMA (FA_S_WARP == FA_PV_WARP).
#ifndef FA_PRODUCER_WARP
#define FA_PRODUCER_WARP 8  // TMA producer
#endif
#ifndef FA_S_WARP
#define FA_S_WARP 10  // issues S = Q K^T
#endif
#ifndef FA_PV_WARP
#define FA_PV_WARP 11  // issues O += P V
#endif
static_assert(FA_PRODUCER_WARP >= 8 && FA_PRODUCER_WARP <= 11 && FA_S_WARP >= 8 &&
                  FA_S_WARP <= 11 && FA_PV_WARP >= 8 && FA_PV_WARP <= 11 &&
                  FA_PRODUCER_WARP != FA_S_WARP && FA_PRODUCER_WARP != FA_PV_WARP,
              "producer and MMA issuers must be distinct warps of warps 8-11");
#ifndef FA_HALVES
#define FA_HALVES 1  // short problems: split each query tile's keys between the warpgroups
#endif
#ifndef FA_SPLIT_MIN_TILES
#define FA_SPLIT_MIN_TILES 8  // fewest key tiles per split of the key-range split mode
#endif
#ifndef FA_EARLY_PASS
#define FA_EARLY_PASS 16  // exponent pairs still to do when the MUFU turn is handed over
#endif

namespace fa {
using namespace ptx;

// Development aid, compiled in only with -DFA_TRACE=1: SM clock stamps of the
// first work item of block 0, written through the debug pointer as
// trace[role][iteration][event] (role 0/1 softmax tile, 2 MMA issuer).
#if FA_TRACE
#define TRACE(role, it, ev)                                                            \
  do {                                                                                 \
    if (p.dbg != nullptr && blockIdx.x == 0 && trace_on && (it) < 64)                   \
      reinterpret_cast<unsigned long long*>(p.dbg)[((role) * 64 + (it)) * 8 + (ev)] =  \
          clock64();                                                                   \
  } while (0)
#else
#define TRACE(role, it, ev) \
  do {                      \
  } while (0)
#endif

constexpr int kHeadDim = 64;
constexpr int kBlockM = 128;   // query rows per tile
constexpr int kBlockN = 128;   // key rows per tile
constexpr int kKvSlots = 6;    // shared-memory ring of 16 KiB K/V tiles
constexpr int kNumThreads = 384;
constexpr uint32_t kTileBytes = kBlockM * kHeadDim * 2;  // 16 KiB, also a K/V tile

constexpr uint32_t kSmemQ = 0;
constexpr uint32_t kSmemKV = kSmemQ + 2 * kTileBytes;
constexpr uint32_t kSmemO = kSmemKV + kKvSlots * kTileBytes;
constexpr uint32_t kSmemCtl = kSmemO + 2 * kTileBytes;
constexpr uint32_t kSmemCtlBytes = 256;
constexpr uint32_t kSmemBytes = kSmemCtl + kSmemCtlBytes + 1024;  // + alignment slack

constexpr uint32_t kTmemCols = 512;
__host__ __device__ constexpr uint32_t col_s(int t) { return t == 0 ? 0u : 128u; }
__host__ __device__ constexpr uint32_t col_o(int t) { return t == 0 ? 256u : 320u; }
__host__ __device__ constexpr uint32_t col_p(int t) { return t == 0 ? 384u : 448u; }

// Status bits written by the kernel (OR-ed into the device status word).
constexpr unsigned int kStatusTimeoutProducer = 1u << 0;
constexpr unsigned int kStatusTimeoutMma = 1u << 1;
constexpr unsigned int kStatusTimeoutSoftmax = 1u << 2;
constexpr unsigned int kStatusTimeoutDrain = 1u << 3;
constexpr unsigned int kStatusTimeoutSelftest = 1u << 4;
// Waits for this block's own copies and MMAs before it exits use their own
// limit, independent of the caller's, so a short limit cannot make a block
// leave with work in flight (those complete within microseconds).
constexpr unsigned long long kDrainLimitNs = 200000000ull;

struct SharedCtl {
  uint64_t q_full, q_empty;
  uint64_t kv_full[kKvSlots], kv_empty[kKvSlots];
  uint64_t s_full[2], s_empty[2], p_full[2], o_done[2], o_empty[2];
  uint64_t exp_turn[2];  // alternates the two softmax warpgroups' exponential phases
  uint64_t wg_bar[2];    // a tile's four softmax warps (key-range split epilogue)
  uint64_t drain[2];     // one per MMA-issuing warp
  uint32_t tmem_base;
  int abort;
  int merge_flag[2];
};
static_assert(sizeof(SharedCtl) <= kSmemCtlBytes, "control block too large");

struct FwdParams {
  int n_q;          // query rows per (batch, head)
  int n_k;          // key/value rows per (batch, head)
  int bh;           // batch * heads
  int causal;       // top-left aligned: key index > query index is masked
  float scale_log2; // softmax scale * log2(e)
  int n_qpairs;     // work items per (batch, head) and split: ceil(ceil(n_q / 128) / 2),
                    // or ceil(n_q / 128) when `single`
  int single;       // 1: a work item is one 128-row query tile (short problems)
  int n_items;      // bh * n_qpairs
  int unit;         // work items per scheduling unit (1 or 2)
  unsigned int* status;
  unsigned long long limit_ns;
  float* dbg;       // optional: first item's first masked score tile (tests)
  float* lse;       // optional: [bh][n_q] row log-sum-exp of the scaled scores (natural log)
  float scale;      // softmax scale (for the log-sum-exp)
  // Key-range split (n_split > 1): a work item is (bh, query pair, split);
  // each split writes fp32 partial results and the last split to finish a
  // query tile merges them.  The three arrays live in one scratch buffer.
  int n_split;      // splits of the key range per query pair (1 = no split)
  int kv_chunk;     // key tiles per split
  int n_qtiles;     // ceil(n_q / 128)
  float* part_o;    // [bh][n_qtiles][n_split][128][64] partial numerators
  float2* part_ml;  // [bh][n_qtiles][n_split][128] (max used, partial sum)
  int* counters;    // [bh][n_qtiles] finished splits; reset to 0 by the merging block
  __half* out;      // o, for the merge's direct stores
};

// Key tiles [jb, n_t[t]) of query tile t belong to the item (n_t[t] <= jb:
// none); n_max = max(n_t).  valid[t]: the query tile exists.
struct ItemShape {
  int bh, qp, split, jb, n_t[2], n_max, q0[2];
  bool valid[2];
};

// Work items are handed out to blocks in units of p.unit consecutive items
// (block b takes units b, b + grid, b + 2 grid, ...), and every role of a
// block walks the same sequence.  Units of two are used when there is more
// than one wave of items; a single wave keeps one item per block.
#define first_item_of_block() (p.unit * static_cast<int>(blockIdx.x))
__device__ __forceinline__ int next_item_of(int item, int unit) {
  if (unit == 1) return item + static_cast<int>(gridDim.x);
  return (item & 1) ? item - 1 + 2 * static_cast<int>(gridDim.x) : item + 1;
}
#define next_item(item) next_item_of(item, p.unit)

template <bool kSplit, bool kHalves = false>
__device__ __forceinline__ ItemShape decode_item(int item, const FwdParams& p) {
  ItemShape s;
  int k;
  if (kSplit) {
    s.split = item % p.n_split;
    const int pair = item / p.n_split;
    s.bh = pair / p.n_qpairs;
    k = pair - s.bh * p.n_qpairs;
  } else {
    s.split = 0;
    s.bh = item / p.n_qpairs;
    k = item - s.bh * p.n_qpairs;
  }
  // Causal work grows with the query position.  Within a head the query
  // pairs are visited as n-1, 0, n-2, 1, ..., so the two items of a unit (a
  // pair and its mirror) always add up to the same amount of work and the
  // static schedule ends balanced.  Both items belong to the same head, which
  // keeps that head's K/V hot in L2.
  s.qp = (p.causal && !kSplit) ? ((k & 1) ? (k >> 1) : (p.n_qpairs - 1 - (k >> 1))) : k;
  const int nkv = (p.n_k + kBlockN - 1) / kBlockN;
  s.jb = kSplit ? s.split * p.kv_chunk : 0;
  const int je = kSplit ? s.jb + p.kv_chunk : 0x7fffffff;
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    s.q0[t] = p.single ? (t == 0 ? s.qp * kBlockM : p.n_q) : s.qp * 2 * kBlockM + t * kBlockM;
    s.valid[t] = s.q0[t] < p.n_q;
    int n = 0;
    if (!s.valid[t]) {
      n = 0;
    } else if (p.causal) {
      const int diag = s.q0[t] / kBlockN + 1;  // tiles up to and including the diagonal
      n = diag < nkv ? diag : nkv;
    } else {
      n = nkv;
    }
    s.n_t[t] = kSplit ? (n < je ? n : je) : n;
  }
  if constexpr (kHalves) {
    // One query tile (p.single); its key tiles are split between the two
    // softmax warpgroups: tile slot 0 takes key tiles [0, n_t[0]), tile slot
    // 1 the rest, [n_t[0], n_t[0] + n_t[1]), against the same query rows.
    const int full = s.n_t[0];
    s.q0[1] = s.q0[0];
    s.valid[1] = false;  // only tile slot 0 writes output
    s.n_t[0] = (full + 1) / 2;
    s.n_t[1] = full - s.n_t[0];
  }
  s.n_max = s.n_t[0] > s.n_t[1] ? s.n_t[0] : s.n_t[1];
  return s;
}

// First key tile of tile slot t (non-zero only for the second half of a
// split key range).
template <bool kHalves>
__device__ __forceinline__ int key_offset(const ItemShape& s, int t) {
  return (kHalves && t == 1) ? s.n_t[0] : 0;
}

// ------------------------------------------------------------------ roles
// Runs on the whole producer warp; one elected lane issues the copies.
template <bool kSplit, bool kHalves>
__device__ bool producer_loop(const FwdParams& p, SharedCtl* ctl, uint32_t smem_base,
                              const CUtensorMap* tm_q, const CUtensorMap* tm_k,
                              const CUtensorMap* tm_v, uint32_t& ld_count, uint32_t& q_count) {
  volatile int* abort_flag = &ctl->abort;
  const uint32_t q_full = smem_u32(&ctl->q_full), q_empty = smem_u32(&ctl->q_empty);
  uint32_t slot = 0, phase = 0;
  for (int item = first_item_of_block(); item < p.n_items; item = next_item(item)) {
    const ItemShape s = decode_item<kSplit, kHalves>(item, p);
    if (s.n_max <= s.jb) continue;  // no key tiles in this item
    if (!mbar_wait_warp(q_empty, (q_count & 1) ^ 1, abort_flag, p.status,
                        kStatusTimeoutProducer, p.limit_ns))
      return false;
    const uint32_t nq = (!kHalves && s.n_t[1] > s.jb) ? 2 : 1;
    if (elect_one()) {
      mbar_arrive_expect_tx(q_full, nq * kTileBytes);
      tma_load_3d(smem_base + kSmemQ, tm_q, q_full, 0, s.q0[0], s.bh);
      if (nq == 2) tma_load_3d(smem_base + kSmemQ + kTileBytes, tm_q, q_full, 0, s.q0[1], s.bh);
    }
    __syncwarp();
    ++q_count;
    for (int j = s.jb; j < s.n_max; ++j) {
      // One K/V pair per step, or with a split key range one per active half
      // (the half's K then V), in the order the MMA warps walk the ring.
#pragma unroll
      for (int g = 0; g < (kHalves ? 2 : 1); ++g) {
        if (kHalves && j >= s.n_t[g]) continue;
        const int kt = key_offset<kHalves>(s, g) + j;
#pragma unroll
        for (int which = 0; which < 2; ++which) {
          if (!mbar_wait_warp(smem_u32(&ctl->kv_empty[slot]), phase ^ 1, abort_flag, p.status,
                              kStatusTimeoutProducer, p.limit_ns))
            return false;
          if (elect_one()) {
            const uint32_t full = smem_u32(&ctl->kv_full[slot]);
            mbar_arrive_expect_tx(full, kTileBytes);
            tma_load_3d(smem_base + kSmemKV + slot * kTileBytes, which ? tm_v : tm_k, full, 0,
                        kt * kBlockN, s.bh);
          }
          __syncwarp();
          ++ld_count;
          if (++slot == kKvSlots) {
            slot = 0;
            phase ^= 1;
          }
        }
      }
    }
  }
  return true;
}

// Runs on a whole MMA warp: waits and bookkeeping are warp-uniform (so the
// descriptors live in uniform registers) and one elected lane issues the
// tcgen05 instructions.  Two warps on different SM sub-partitions share the
// work (kIssueS: S_t = Q_t K_j^T; kIssuePV: O_t += P_t V_j), because issuing
// tcgen05.mma slows the softmax warps on the issuing sub-partition.  Per key
// tile j the order is S_0(j), S_1(j), then O_0 += P_0(j-1) V_{j-1},
// O_1 += P_1(j-1) V_{j-1}.
template <bool kSplit, bool kIssueS, bool kIssuePV>
__device__ bool mma_loop(const FwdParams& p, SharedCtl* ctl, uint32_t smem_base,
                         uint32_t tmem) {
  volatile int* abort_flag = &ctl->abort;
  constexpr uint32_t idesc_qk = idesc_f16_f32(kBlockM, kBlockN, false);
  constexpr uint32_t idesc_pv = idesc_f16_f32(kBlockM, kHeadDim, true);
  uint32_t slot = 0, phase = 0;  // ring position of the next K tile
  uint32_t q_count = 0;
  uint32_t s_cnt[2] = {0, 0}, p_cnt[2] = {0, 0}, o_cnt[2] = {0, 0};
  // Descriptor bases; the start-address field (bits 0-13, 16-byte units) is
  // advanced by plain addition: every operand lies below 256 KiB.
  const uint64_t dq0 = smem_desc_sw128(smem_base + kSmemQ, 16, 1024);
  const uint64_t dkv = smem_desc_sw128(smem_base + kSmemKV, 16, 1024);
  constexpr uint64_t kTileDesc = kTileBytes >> 4;

  auto wait = [&](uint32_t bar, uint32_t parity) {
    return mbar_wait_warp(bar, parity, abort_flag, p.status, kStatusTimeoutMma, p.limit_ns);
  };

  for (int item = first_item_of_block(); item < p.n_items; item = next_item(item)) {
    const ItemShape s = decode_item<kSplit>(item, p);
    if (s.n_max <= s.jb) continue;  // no key tiles in this item
    if (kIssueS) {
      if (!wait(smem_u32(&ctl->q_full), q_count & 1)) return false;
      ++q_count;
      tc_fence_after();
    }
    uint32_t v_slot = 0, v_phase = 0;  // ring position of V_{j-1}
    const bool trace_on = item == first_item_of_block() && threadIdx.x % 32 == 0;
    (void)trace_on;
    for (int j = s.jb; j <= s.n_max; ++j) {
      TRACE(2, j, 0);
      uint32_t next_v_slot = 0, next_v_phase = 0;
      const uint32_t ks = slot, kph = phase;  // ring position of K_j
      if (j < s.n_max) {
        next_v_slot = ks + 1 == kKvSlots ? 0 : ks + 1;
        next_v_phase = ks + 1 == kKvSlots ? kph ^ 1 : kph;
        slot += 2;  // past K_j and V_j
        if (slot >= kKvSlots) {
          slot -= kKvSlots;
          phase ^= 1;
        }
      }
      if (kIssueS && j < s.n_max) {
        // ---- S_t = Q_t K_j^T for every tile that still needs key tile j
        if (!wait(smem_u32(&ctl->kv_full[ks]), kph)) return false;
        TRACE(2, j, 1);
        tc_fence_after();
        const uint64_t dk = dkv + ks * kTileDesc;
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          if (j >= s.n_t[t]) continue;
          if (!wait(smem_u32(&ctl->s_empty[t]), (s_cnt[t] & 1) ^ 1)) return false;
          ++s_cnt[t];
          if (t == 0) TRACE(2, j, 2);
          tc_fence_after();
          if (elect_one()) {
            const uint64_t dq = dq0 + t * kTileDesc;
#pragma unroll
            for (int kk = 0; kk < kHeadDim / 16; ++kk)  // 16 dims = 32 bytes per step
              mma_ss_f16(tmem + col_s(t), dq + 2 * kk, dk + 2 * kk, idesc_qk, kk > 0);
            tc_commit(smem_u32(&ctl->s_full[t]));
          }
          __syncwarp();
          TRACE(2, j, 3 + t);
        }
        if (elect_one()) {
          tc_commit(smem_u32(&ctl->kv_empty[ks]));
          if (j == s.n_max - 1) tc_commit(smem_u32(&ctl->q_empty));
        }
        __syncwarp();
      }
      if (kIssuePV && j > s.jb) {
        // ---- O_t += P_t V_{j-1}
        const int jj = j - 1;
        if (!wait(smem_u32(&ctl->kv_full[v_slot]), v_phase)) return false;
        TRACE(2, j, 5);
        tc_fence_after();
        const uint64_t dv = dkv + v_slot * kTileDesc;
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          if (jj >= s.n_t[t]) continue;
          if (jj == s.jb) {
            // O_t is overwritten by this item's first PV: the previous item's
            // epilogue must have read it.
            if (!wait(smem_u32(&ctl->o_empty[t]), (o_cnt[t] & 1) ^ 1)) return false;
            ++o_cnt[t];
          }
          if (!wait(smem_u32(&ctl->p_full[t]), p_cnt[t] & 1)) return false;
          ++p_cnt[t];
          if (t == 0) TRACE(2, j, 6);
          tc_fence_after();
          if (elect_one()) {
#pragma unroll
            for (int kk = 0; kk < kBlockN / 16; ++kk) {
              // P: 16 keys = 8 packed columns per step; V: 16 key rows = 2 KiB.
              mma_ts_f16(tmem + col_o(t), tmem + col_p(t) + kk * 8, dv + 128 * kk, idesc_pv,
                         (jj > s.jb || kk > 0) ? 1u : 0u);
            }
            tc_commit(smem_u32(&ctl->o_done[t]));
          }
          __syncwarp();
          if (t == 0) TRACE(2, j, 7);
        }
        if (elect_one()) tc_commit(smem_u32(&ctl->kv_empty[v_slot]));
        __syncwarp();
      }
      v_slot = next_v_slot;
      v_phase = next_v_phase;
    }
  }
  return true;
}

// MMA issue for items whose single query tile has its key range split
// between the two tile slots (short problems): slot t computes
// S_t = Q K_{o_t + j}^T and O_t += P_t V_{o_t + j} with o_0 = 0 and
// o_1 = n_t[0], both against the one Q tile.  Per step the ring holds K, V of
// slot 0 and then K, V of slot 1 (when active), as the producer loads them.
template <bool kIssueS, bool kIssuePV>
__device__ bool mma_loop_halves(const FwdParams& p, SharedCtl* ctl, uint32_t smem_base,
                                uint32_t tmem) {
  volatile int* abort_flag = &ctl->abort;
  constexpr uint32_t idesc_qk = idesc_f16_f32(kBlockM, kBlockN, false);
  constexpr uint32_t idesc_pv = idesc_f16_f32(kBlockM, kHeadDim, true);
  uint32_t slot = 0, phase = 0;
  uint32_t q_count = 0;
  uint32_t s_cnt[2] = {0, 0}, p_cnt[2] = {0, 0}, o_cnt[2] = {0, 0};
  const uint64_t dq = smem_desc_sw128(smem_base + kSmemQ, 16, 1024);
  const uint64_t dkv = smem_desc_sw128(smem_base + kSmemKV, 16, 1024);
  constexpr uint64_t kTileDesc = kTileBytes >> 4;

  auto wait = [&](uint32_t bar, uint32_t parity) {
    return mbar_wait_warp(bar, parity, abort_flag, p.status, kStatusTimeoutMma, p.limit_ns);
  };

  for (int item = first_item_of_block(); item < p.n_items; item = next_item(item)) {
    const ItemShape s = decode_item<false, true>(item, p);
    if (s.n_max <= 0) continue;
    if (kIssueS) {
      if (!wait(smem_u32(&ctl->q_full), q_count & 1)) return false;
      ++q_count;
      tc_fence_after();
    }
    uint32_t v_slot[2] = {0, 0}, v_phase[2] = {0, 0};  // ring position of V of the last step
    for (int j = 0; j <= s.n_max; ++j) {
      uint32_t nv_slot[2] = {0, 0}, nv_phase[2] = {0, 0};
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        if (j >= s.n_t[t]) continue;
        const uint32_t ks = slot, kph = phase;
        nv_slot[t] = ks + 1 == kKvSlots ? 0 : ks + 1;
        nv_phase[t] = ks + 1 == kKvSlots ? kph ^ 1 : kph;
        slot += 2;  // past this slot's K and V
        if (slot >= kKvSlots) {
          slot -= kKvSlots;
          phase ^= 1;
        }
        if (kIssueS) {
          // ---- S_t = Q K_{o_t + j}^T
          if (!wait(smem_u32(&ctl->kv_full[ks]), kph)) return false;
          if (!wait(smem_u32(&ctl->s_empty[t]), (s_cnt[t] & 1) ^ 1)) return false;
          ++s_cnt[t];
          tc_fence_after();
          if (elect_one()) {
            const uint64_t dk = dkv + ks * kTileDesc;
#pragma unroll
            for (int kk = 0; kk < kHeadDim / 16; ++kk)
              mma_ss_f16(tmem + col_s(t), dq + 2 * kk, dk + 2 * kk, idesc_qk, kk > 0);
            tc_commit(smem_u32(&ctl->s_full[t]));
            tc_commit(smem_u32(&ctl->kv_empty[ks]));
          }
          __syncwarp();
        }
      }
      if (kIssueS && j == s.n_max - 1) {
        if (elect_one()) tc_commit(smem_u32(&ctl->q_empty));
        __syncwarp();
      }
      if (kIssuePV && j > 0) {
        // ---- O_t += P_t V_{o_t + j - 1}
        const int jj = j - 1;
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          if (jj >= s.n_t[t]) continue;
          if (!wait(smem_u32(&ctl->kv_full[v_slot[t]]), v_phase[t])) return false;
          if (jj == 0) {
            // O_t is overwritten by this item's first PV: the previous item's
            // epilogue must have read it.
            if (!wait(smem_u32(&ctl->o_empty[t]), (o_cnt[t] & 1) ^ 1)) return false;
            ++o_cnt[t];
          }
          if (!wait(smem_u32(&ctl->p_full[t]), p_cnt[t] & 1)) return false;
          ++p_cnt[t];
          tc_fence_after();
          if (elect_one()) {
            const uint64_t dv = dkv + v_slot[t] * kTileDesc;
#pragma unroll
            for (int kk = 0; kk < kBlockN / 16; ++kk)
              mma_ts_f16(tmem + col_o(t), tmem + col_p(t) + kk * 8, dv + 128 * kk, idesc_pv,
                         (jj > 0 || kk > 0) ? 1u : 0u);
            tc_commit(smem_u32(&ctl->o_done[t]));
            tc_commit(smem_u32(&ctl->kv_empty[v_slot[t]]));
          }
          __syncwarp();
        }
      }
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        v_slot[t] = nv_slot[t];
        v_phase[t] = nv_phase[t];
      }
    }
  }
  return true;
}

template <bool kSplit, bool kTurnsAlways, bool kHalves, bool kLse>
__device__ bool softmax_loop(const FwdParams& p, SharedCtl* ctl, uint32_t smem_base,
                             uint32_t tmem, const CUtensorMap* tm_o, int t, int warp_in_group,
                             int lane) {
  volatile int* abort_flag = &ctl->abort;
  const int row = warp_in_group * 32 + lane;
  const uint32_t lane_base = static_cast<uint32_t>(warp_in_group * 32) << 16;
  const uint32_t t_s = tmem + lane_base + col_s(t);
  const uint32_t t_o = tmem + lane_base + col_o(t);
  const uint32_t t_p = tmem + lane_base + col_p(t);
  const uint32_t s_full = smem_u32(&ctl->s_full[t]);
  const uint32_t s_empty = smem_u32(&ctl->s_empty[t]);
  const uint32_t p_full = smem_u32(&ctl->p_full[t]);
  const uint32_t o_done = smem_u32(&ctl->o_done[t]);
  const uint32_t o_empty = smem_u32(&ctl->o_empty[t]);
  const uint32_t stage = smem_base + kSmemO + t * kTileBytes;
  const float c = p.scale_log2;
  uint32_t s_cnt = 0, od_cnt = 0, wg_cnt = 0;
  uint32_t merge_cnt = 0;  // items merged (split key range within the block)

  auto wait = [&](uint32_t bar, uint32_t parity) {
    return mbar_wait_warp(bar, parity, abort_flag, p.status, kStatusTimeoutSoftmax,
                          p.limit_ns);
  };

  // The exponentials of both tiles share the SM's MUFU units (16 ex2/clk).
  // The two warpgroups take turns (tile 0, tile 1, tile 0, ...), so one's
  // exponentials overlap the other's P store, S load and row max.  Both run
  // n_max rounds per work item; a tile with fewer key tiles (or none) passes
  // its extra turns without work.
  const uint32_t turn_mine = smem_u32(&ctl->exp_turn[t]);
  const uint32_t turn_other = smem_u32(&ctl->exp_turn[t ^ 1]);
  uint32_t turn_cnt = 0;
  // Turns are taken only in items where both tiles have key tiles; a lone
  // tile runs freely.
  bool use_turns = true;  // constant in kernels whose items all have two tiles
  auto take_turn = [&]() {
    if (!use_turns) return true;
    return wait(turn_mine, (turn_cnt & 1) ^ (t == 0 ? 1u : 0u));
  };
  auto pass_turn = [&]() {
    if (!use_turns) return;
    __syncwarp();
    if (lane == 0) mbar_arrive(turn_other);
    ++turn_cnt;
  };

  // Barrier of the tile's four softmax warps, bounded like every other wait
  // (a named barrier would wait forever for a warp that gave up).
  auto wg_sync = [&]() {
    const uint32_t bar = smem_u32(&ctl->wg_bar[t]);
    __syncwarp();
    if (lane == 0) mbar_arrive(bar);
    const bool ok = wait(bar, wg_cnt & 1);
    ++wg_cnt;
    return ok;
  };

  // Key-range split epilogue: store this split's partial result (numerator
  // rows `orr`, or none for an empty range, with the max used and the partial
  // sum), count the split as finished, and let the last split of the query
  // tile merge all partials into o.
  auto split_epilogue = [&](const ItemShape& s, const uint32_t* orr, float m, float lsum) {
    const int qtile = s.q0[t] / kBlockM;
    const size_t tile_idx = static_cast<size_t>(s.bh) * p.n_qtiles + qtile;
    const size_t part = (tile_idx * p.n_split + s.split) * kBlockM + row;
    if (orr != nullptr) {
      float4* dst = reinterpret_cast<float4*>(p.part_o + part * kHeadDim);
#pragma unroll
      for (int i = 0; i < 16; ++i)
        dst[i] = make_float4(__uint_as_float(orr[4 * i]), __uint_as_float(orr[4 * i + 1]),
                             __uint_as_float(orr[4 * i + 2]), __uint_as_float(orr[4 * i + 3]));
    }
    p.part_ml[part] = make_float2(m, lsum);
    __threadfence();
    if (!wg_sync()) return false;
    if (row == 0) {
      const int done = atomicAdd(p.counters + tile_idx, 1) + 1;
      const int last = done == p.n_split ? 1 : 0;
      if (last) {
        atomicExch(p.counters + tile_idx, 0);  // ready for the next launch
        __threadfence();
      }
      ctl->merge_flag[t] = last;
    }
    if (!wg_sync()) return false;
    if (!*reinterpret_cast<volatile int*>(&ctl->merge_flag[t])) return true;
    // ---- merge: o = sum_s w_s O_s / sum_s w_s l_s, w_s = 2^((m_s - max m) * c)
    const size_t base = tile_idx * p.n_split * kBlockM + row;
    float mmax = -INFINITY;
    for (int sp = 0; sp < p.n_split; ++sp) {
      const float2 ml = __ldcg(p.part_ml + base + static_cast<size_t>(sp) * kBlockM);
      if (ml.y > 0.f) mmax = fmaxf(mmax, ml.x);
    }
    float acc[kHeadDim];
#pragma unroll
    for (int i = 0; i < kHeadDim; ++i) acc[i] = 0.f;
    float den = 0.f;
    for (int sp = 0; sp < p.n_split; ++sp) {
      const size_t pi = base + static_cast<size_t>(sp) * kBlockM;
      const float2 ml = __ldcg(p.part_ml + pi);
      if (!(ml.y > 0.f)) continue;
      const float w = ex2_approx((ml.x - mmax) * c);
      den = fmaf(w, ml.y, den);
      const float4* src = reinterpret_cast<const float4*>(p.part_o + pi * kHeadDim);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float4 v = __ldcg(src + i);
        acc[4 * i] = fmaf(w, v.x, acc[4 * i]);
        acc[4 * i + 1] = fmaf(w, v.y, acc[4 * i + 1]);
        acc[4 * i + 2] = fmaf(w, v.z, acc[4 * i + 2]);
        acc[4 * i + 3] = fmaf(w, v.w, acc[4 * i + 3]);
      }
    }
    const int qr = s.q0[t] + row;
    if constexpr (kLse) {
      if (qr < p.n_q) p.lse[static_cast<size_t>(s.bh) * p.n_q + qr] = mmax * p.scale + logf(den);
    }
    if (qr < p.n_q) {
      const float inv = 1.f / den;
      uint4* dst = reinterpret_cast<uint4*>(p.out + (static_cast<size_t>(s.bh) * p.n_q + qr) *
                                                        kHeadDim);
#pragma unroll
      for (int i = 0; i < 8; ++i)
        dst[i] = make_uint4(pack_half2(acc[8 * i] * inv, acc[8 * i + 1] * inv),
                            pack_half2(acc[8 * i + 2] * inv, acc[8 * i + 3] * inv),
                            pack_half2(acc[8 * i + 4] * inv, acc[8 * i + 5] * inv),
                            pack_half2(acc[8 * i + 6] * inv, acc[8 * i + 7] * inv));
    }
    return true;
  };

  for (int item = first_item_of_block(); item < p.n_items; item = next_item(item)) {
    const ItemShape s = decode_item<kSplit, kHalves>(item, p);
    const int n_t = s.n_t[t];
    use_turns = kTurnsAlways || (s.n_t[0] > s.jb && s.n_t[1] > s.jb);
    if (!kHalves && n_t <= s.jb) {
      for (int j = s.jb; j < s.n_max; ++j) {
        if (!take_turn()) return false;
        pass_turn();
      }
      if constexpr (kSplit) {
        if (s.valid[t] && !split_epilogue(s, nullptr, -INFINITY, 0.f)) return false;
      }
      continue;
    }
    const int q_row = s.q0[t] + row;
    float m_used = -INFINITY;
    float l = 0.f;

    for (int j = s.jb; j < n_t; ++j) {
      const bool trace_on = item == first_item_of_block() && row == 0;
      (void)trace_on;
      TRACE(t, j, 0);
      if (!wait(s_full, s_cnt & 1)) return false;
      TRACE(t, j, 1);
      ++s_cnt;
      tc_fence_after();
      uint32_t sr[128];
#pragma unroll
      for (int i = 0; i < 4; ++i) tmem_ld32(t_s + 32 * i, sr + 32 * i);
      tc_wait_ld();
      TRACE(t, j, 2);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(s_empty);

      const int kv0 = (key_offset<kHalves>(s, t) + j) * kBlockN;
      const bool need_mask =
          (p.causal && kv0 + kBlockN - 1 > s.q0[t]) || (kv0 + kBlockN > p.n_k);
      if (need_mask) {
        const int lim_causal = p.causal ? (q_row - kv0) : (kBlockN - 1);
        const int lim_tail = p.n_k - kv0 - 1;
        const int lim = lim_causal < lim_tail ? lim_causal : lim_tail;
#pragma unroll
        for (int i = 0; i < 128; ++i)
          if (i > lim) sr[i] = __float_as_uint(-INFINITY);
      }
      if (!FA_TRACE && p.dbg != nullptr && item == first_item_of_block() &&
          blockIdx.x == 0 && j == 0) {
#pragma unroll
        for (int i = 0; i < 128; ++i) p.dbg[(t * 128 + row) * 128 + i] = __uint_as_float(sr[i]);
      }

      // Row max: eight independent chains of three-input maxima.
      float mx[8];
#pragma unroll
      for (int a = 0; a < 8; ++a) {
        const uint32_t* g = sr + 16 * a;
        float acc = max3f(__uint_as_float(g[0]), __uint_as_float(g[1]), __uint_as_float(g[2]));
#pragma unroll
        for (int e = 3; e + 1 < 16; e += 2)
          acc = max3f(acc, __uint_as_float(g[e]), __uint_as_float(g[e + 1]));
        mx[a] = fmaxf(acc, __uint_as_float(g[15]));
      }
      const float m_new = max3f(max3f(mx[0], mx[1], mx[2]), max3f(mx[3], mx[4], mx[5]),
                                max3f(mx[6], mx[7], m_used));
      TRACE(t, j, 3);
      const bool rescale = (m_new - m_used) * c > 8.0f;
      float alpha = 1.f;
      if (rescale) {
        alpha = ex2_approx((m_used - m_new) * c);
        m_used = m_new;
        l *= alpha;
      }
      const float neg = -m_used * c;
      if (!take_turn()) return false;
      TRACE(t, j, 7);

      // p = 2^(s*c - m*c): packed FMA for the exponent, MUFU ex2, packed sums
      // in eight independent chains, fp16 pairs kept in registers until P_t is
      // free again.
      uint32_t pk[64];
      float sum[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int i = 0; i < 64; ++i) {
        if (i == 64 - FA_EARLY_PASS) pass_turn();
        float x0, x1;
        ffma2(x0, x1, __uint_as_float(sr[2 * i]), __uint_as_float(sr[2 * i + 1]), c, c, neg, neg);
        float p0, p1;
        if ((i & 7) < FA_POLY_PAIRS) {
          exp2_poly2(p0, p1, x0, x1);
        } else {
          p0 = ex2_approx(x0);
          p1 = ex2_approx(x1);
        }
        const int a = (i & 3) * 2;
        fadd2(sum[a], sum[a + 1], sum[a], sum[a + 1], p0, p1);
        pk[i] = pack_half2(p0, p1);
      }
      if (FA_EARLY_PASS == 0) pass_turn();
      l += ((sum[0] + sum[1]) + (sum[2] + sum[3])) + ((sum[4] + sum[5]) + (sum[6] + sum[7]));
      TRACE(t, j, 4);

      if (j > s.jb) {
        // PV(j-1) must be done before P_t is overwritten or O_t is rescaled.
        if (!wait(o_done, od_cnt & 1)) return false;
        ++od_cnt;
        TRACE(t, j, 5);
        tc_fence_after();
        if (__any_sync(0xffffffffu, rescale)) {
          uint32_t orr[64];
          tmem_ld32(t_o, orr);
          tmem_ld32(t_o + 32, orr + 32);
          tc_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            float a0, a1;
            fmul2(a0, a1, __uint_as_float(orr[2 * i]), __uint_as_float(orr[2 * i + 1]), alpha,
                  alpha);
            orr[2 * i] = __float_as_uint(a0);
            orr[2 * i + 1] = __float_as_uint(a1);
          }
          tmem_st32(t_o, orr);
          tmem_st32(t_o + 32, orr + 32);
        }
      }
      tmem_st32(t_p, pk);
      tmem_st32(t_p + 32, pk + 32);
      tc_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
      TRACE(t, j, 6);
    }

    for (int j = n_t; j < s.n_max; ++j) {
      if (!take_turn()) return false;
      pass_turn();
    }

    // ---- epilogue: O / l -> fp16 -> swizzled staging tile -> TMA store
    if (!kHalves || n_t > 0) {
      if (!wait(o_done, od_cnt & 1)) return false;  // the last P V of this tile slot
      ++od_cnt;
    }
    uint32_t orr[64];
    if constexpr (kHalves) {
      // The two tile slots hold the same query rows over two halves of the
      // key range.  Slot 1 hands its (max used, sum) to slot 0 through
      // shared memory (the unused output staging tile of slot 1); slot 0
      // reads both partial numerators from tensor memory and merges:
      // m = max(m0, m1), O = O0 2^((m0-m)c) + O1 2^((m1-m)c), likewise l.
      float* ml = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(ctl) - kSmemCtl + kSmemO +
                                           kTileBytes);
      const uint32_t ml_free = smem_u32(&ctl->wg_bar[0]);   // slot 0 has read (m, l)
      const uint32_t ml_ready = smem_u32(&ctl->wg_bar[1]);  // slot 1 has written them
      if (t == 1) {
        if (!wait(ml_free, (merge_cnt & 1) ^ 1)) return false;
        ++merge_cnt;
        ml[row] = n_t > 0 ? m_used : -INFINITY;
        ml[kBlockM + row] = n_t > 0 ? l : 0.f;
        __syncwarp();
        if (lane == 0) mbar_arrive(ml_ready);
        continue;
      }
      if (!wait(ml_ready, merge_cnt & 1)) return false;
      ++merge_cnt;
      tc_fence_after();
      const float m1 = ml[row], l1 = ml[kBlockM + row];
      __syncwarp();
      if (lane == 0) mbar_arrive(ml_free);
      tmem_ld32(t_o, orr);
      tmem_ld32(t_o + 32, orr + 32);
      tc_wait_ld();
      const bool other = s.n_t[1] > 0;
      if (other) {
        const float m = fmaxf(m_used, m1);
        const float w0 = ex2_approx((m_used - m) * c), w1 = ex2_approx((m1 - m) * c);
        l = l * w0 + l1 * w1;
        m_used = m;
        const uint32_t t_o1 = tmem + lane_base + col_o(1);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint32_t o1[32];
          tmem_ld32(t_o1 + 32 * h, o1);
          tc_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i)
            orr[32 * h + i] = __float_as_uint(
                fmaf(__uint_as_float(orr[32 * h + i]), w0, __uint_as_float(o1[i]) * w1));
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(o_empty);
        if (other) mbar_arrive(smem_u32(&ctl->o_empty[1]));
      }
    } else {
      tc_fence_after();
      tmem_ld32(t_o, orr);
      tmem_ld32(t_o + 32, orr + 32);
      tc_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(o_empty);
    }
    if constexpr (kSplit) {
      if (!split_epilogue(s, orr, m_used, l)) return false;
      continue;
    }

    const float inv = 1.f / l;
    if constexpr (kLse) {
      const int qr = s.q0[t] + row;
      if (qr < p.n_q) p.lse[static_cast<size_t>(s.bh) * p.n_q + qr] = m_used * p.scale + logf(l);
    }
    uint32_t h[32];
#pragma unroll
    for (int i = 0; i < 32; ++i)
      h[i] = pack_half2(__uint_as_float(orr[2 * i]) * inv, __uint_as_float(orr[2 * i + 1]) * inv);

    // Each warp stores its own 32 rows: a 4 KiB slice of the staging tile
    // and one TMA store, so the epilogue needs no warpgroup barrier.  The
    // slice is rewritten only after this warp's previous store has read it.
    if (lane == 0) bulk_wait_group_read0();
    __syncwarp();
    const uint32_t row_addr = stage + row * 128;
#pragma unroll
    for (int ch = 0; ch < 8; ++ch) {
      const uint32_t dst = row_addr + ((ch ^ (row & 7)) << 4);
      asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(dst), "r"(h[4 * ch]),
                   "r"(h[4 * ch + 1]), "r"(h[4 * ch + 2]), "r"(h[4 * ch + 3])
                   : "memory");
    }
    fence_proxy_async_smem();
    __syncwarp();
    const int warp_row0 = s.q0[t] + warp_in_group * 32;
    if (lane == 0 && warp_row0 < p.n_q) {
      tma_store_3d(tm_o, stage + warp_in_group * 32 * 128, 0, warp_row0, s.bh);
      bulk_commit_group();
    }
  }
  return true;
}

// kSplit: key-range split items (fp32 partials, merged by the last split).
// kTurnsAlways: every item has two query tiles with key tiles, so the MUFU
// turns are never skipped.  kHalves: one query tile per item whose key range
// is split between the two softmax warpgroups and merged in the block (short
// problems).  Separate instantiations keep the split merge and the per-item
// turn check out of the main path's code.
template <bool kSplit, bool kTurnsAlways, bool kHalves, bool kLse = false>
__global__ void __launch_bounds__(kNumThreads, 1)
    fa_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                  const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
                  const FwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t smem_base = (raw + 1023u) & ~1023u;  // SW128 tiles need 1 KiB alignment
  SharedCtl* ctl = reinterpret_cast<SharedCtl*>(smem_raw + (smem_base - raw) + kSmemCtl);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&ctl->q_full), 1);
    mbar_init(smem_u32(&ctl->q_empty), 1);
    for (int i = 0; i < kKvSlots; ++i) {
      mbar_init(smem_u32(&ctl->kv_full[i]), 1);
      mbar_init(smem_u32(&ctl->kv_empty[i]), 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(smem_u32(&ctl->s_full[t]), 1);
      mbar_init(smem_u32(&ctl->s_empty[t]), 4);
      mbar_init(smem_u32(&ctl->p_full[t]), 4);
      mbar_init(smem_u32(&ctl->o_done[t]), 1);
      mbar_init(smem_u32(&ctl->o_empty[t]), 4);
      mbar_init(smem_u32(&ctl->exp_turn[t]), 4);
      mbar_init(smem_u32(&ctl->wg_bar[t]), 4);
    }
    mbar_init(smem_u32(&ctl->drain[0]), 1);
    mbar_init(smem_u32(&ctl->drain[1]), 1);
    ctl->abort = 0;
    fence_mbar_init();
  }
  if (warp == FA_PRODUCER_WARP && lane == 0) {
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
    tma_prefetch_desc(&tm_o);
  }
  if (warp == 9) {
    tmem_alloc(smem_u32(&ctl->tmem_base), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;

  if (warp < 8) {
    // Softmax warpgroups take the registers the producer/MMA warpgroup gives
    // up: 2 x 128 x 208 + 128 x 88 = 384 x 168 (the launch allocation).
    asm volatile("setmaxnreg.inc.sync.aligned.u32 208;" ::: "memory");
    const bool ok =
        softmax_loop<kSplit, kTurnsAlways, kHalves, kLse>(p, ctl, smem_base, tmem, &tm_o, warp / 4,
                                                    warp % 4, lane);
    (void)ok;
    if (lane == 0) bulk_wait_group0();  // this warp's output stores
  } else {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 88;" ::: "memory");
  }
  if (warp == FA_PRODUCER_WARP) {
    uint32_t ld_count = 0, q_count = 0;
    const bool ok = producer_loop<kSplit, kHalves>(p, ctl, smem_base, &tm_q, &tm_k, &tm_v,
                                                   ld_count, q_count);
    if (!ok && lane == 0) {
      // Let every copy this warp started land before the block exits.
      const uint32_t n = ld_count < kKvSlots ? ld_count : kKvSlots;
      for (uint32_t i = 0; i < n; ++i) {
        const uint32_t idx = ld_count - 1 - i;
        mbar_wait(smem_u32(&ctl->kv_full[idx % kKvSlots]), (idx / kKvSlots) & 1, nullptr,
                  p.status, kStatusTimeoutDrain, kDrainLimitNs);
      }
      if (q_count > 0)
        mbar_wait(smem_u32(&ctl->q_full), (q_count - 1) & 1, nullptr, p.status,
                  kStatusTimeoutDrain, kDrainLimitNs);
    }
    __syncwarp();
  } else if (warp == FA_S_WARP || warp == FA_PV_WARP) {
    if (warp == FA_S_WARP) {
      if constexpr (kHalves)
        mma_loop_halves<true, FA_S_WARP == FA_PV_WARP>(p, ctl, smem_base, tmem);
      else
        mma_loop<kSplit, true, FA_S_WARP == FA_PV_WARP>(p, ctl, smem_base, tmem);
    } else {
      if constexpr (kHalves)
        mma_loop_halves<false, true>(p, ctl, smem_base, tmem);
      else
        mma_loop<kSplit, false, true>(p, ctl, smem_base, tmem);
    }
    // Every MMA this warp issued (and the barrier arrivals its commits
    // perform) finishes before tensor memory and shared memory are released.
    const uint32_t drain = smem_u32(&ctl->drain[warp == FA_S_WARP ? 0 : 1]);
    if (lane == 0) {
      tc_commit(drain);
      mbar_wait(drain, 0, nullptr, p.status, kStatusTimeoutDrain, kDrainLimitNs);
    }
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

__global__ void selftest_timeout_kernel(unsigned int* status, unsigned long long limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    abort_flag = 0;
    mbar_init(smem_u32(&bar), 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // Nothing ever arrives on this barrier: the wait must give up by itself.
    mbar_wait(smem_u32(&bar), 0, &abort_flag, status, kStatusTimeoutSelftest, limit_ns);
  }
}

__device__ unsigned int g_status_word;

}  // namespace fa

#include "fa_bwd_sm100.cuh"

namespace fa {

// Scratch of fa_fwd_sm100_noalloc: a fixed array that exists on every device
// that loads this library, for callers that cannot allocate.  12 MiB covers
// the largest key-range split plan on a 148-SM B200 (at most ~296 partial
// query tiles of 33 KiB plus the counter prefix).
constexpr size_t kNoAllocScratchBytes = 12u << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

}  // namespace fa

// ====================================================================== host
namespace {

thread_local char g_last_error[512] = "";
// Process-wide policy, set by fa_set_wait_limit_ns / fa_set_max_splits from
// any thread and read by every launch.
constexpr unsigned long long kDefaultWaitLimitNs = 2000000000ull;  // 2 s
std::atomic<unsigned long long> g_wait_limit_ns{kDefaultWaitLimitNs};

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

constexpr int kMaxDevices = 64;
struct DeviceState {
  bool ready = false;
  int sms = 0;
  unsigned int* status = nullptr;
  void* noalloc_scratch = nullptr;  // device address of g_noalloc_scratch
};
DeviceState g_dev[kMaxDevices];
EncodeTiledFn g_encode = nullptr;
std::mutex g_mutex;
std::atomic<int> g_max_splits{0};  // 0: automatic, 1: never split the key range, k: at most k splits

// Scratch of the key-range split mode, one buffer per (device, stream) so
// launches on different streams never share it; launches on one stream are
// ordered.  Allocated on first need, grown when a larger problem arrives, and
// held until fa_release_workspaces() (also for streams destroyed since).  The
// map is guarded by g_mutex only while an entry is looked up; the device calls
// that grow a buffer hold that entry's own mutex, so one stream's allocation
// never blocks another stream's launch.
struct Workspace {
  std::mutex mu;
  void* ptr = nullptr;
  size_t bytes = 0;
};
std::map<std::pair<int, cudaStream_t>, std::unique_ptr<Workspace>> g_workspaces;

// How a launch splits the key range, and the scratch that needs.
struct SplitPlan {
  int n_split = 1, kv_chunk = 0, n_qtiles = 0;
  size_t counters_bytes = 0, ml_bytes = 0, o_bytes = 0;
  size_t total() const { return counters_bytes + ml_bytes + o_bytes; }
};

size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

// The split counters occupy a fixed prefix of every scratch buffer, whatever
// the problem, so the partial results of one launch never land where another
// launch's counters live: the kernel leaves every counter it uses at zero and
// nothing else writes to the prefix.
constexpr size_t kMaxSplitTiles = 1024;
constexpr size_t kCounterBytes = kMaxSplitTiles * sizeof(int);

SplitPlan plan_split(int64_t bh, int64_t n_q, int64_t n_k, int sms) {
  SplitPlan sp;
  const int max_splits = g_max_splits.load(std::memory_order_relaxed);
  const int64_t n_qpairs = ((n_q + 127) / 128 + 1) / 2;
  const int64_t pairs = bh * n_qpairs;
  const int64_t nkv = (n_k + 127) / 128;
  sp.n_qtiles = static_cast<int>((n_q + 127) / 128);
  sp.kv_chunk = static_cast<int>(nkv);
  // Split only when the query pairs leave SMs idle, and keep >= 8 key tiles
  // per split: a block's fixed cost (Q load, pipeline fill, partial write and
  // merge) is worth a few key tiles, so shorter splits measured slower than
  // no split on a B200.
  // Automatic policy: query tiles that fit in one wave go to one block each,
  // with the key range split between the block's two softmax warpgroups and
  // merged in the block (no scratch); measured faster than splitting across
  // blocks for every such shape on a B200.  An explicit split limit (> 1)
  // still selects the cross-block split.
  const bool one_wave_halves = FA_HALVES && max_splits == 0 && bh * sp.n_qtiles <= sms;
  if (max_splits != 1 && pairs < sms && !one_wave_halves) {
    int64_t want = sms / pairs;
    const int64_t cap = nkv / FA_SPLIT_MIN_TILES;
    if (want > cap) want = cap;
    if (max_splits > 1 && want > max_splits) want = max_splits;
    if (want >= 2) {
      sp.kv_chunk = static_cast<int>((nkv + want - 1) / want);
      sp.n_split = static_cast<int>((nkv + sp.kv_chunk - 1) / sp.kv_chunk);
    }
  }
  if (sp.n_split > 1 && static_cast<size_t>(bh) * sp.n_qtiles > kMaxSplitTiles) {
    sp.n_split = 1;
    sp.kv_chunk = static_cast<int>(nkv);
  }
  if (sp.n_split > 1) {
    const size_t tiles = static_cast<size_t>(bh) * sp.n_qtiles;
    sp.counters_bytes = kCounterBytes;
    sp.ml_bytes = align256(tiles * sp.n_split * 128 * sizeof(float2));
    sp.o_bytes = tiles * sp.n_split * 128 * 64 * sizeof(float);
  }
  return sp;
}

int get_workspace(int dev, cudaStream_t stream, size_t need, void** out) {
  Workspace* w = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_mutex);
    std::unique_ptr<Workspace>& slot = g_workspaces[std::make_pair(dev, stream)];
    if (!slot) slot.reset(new Workspace());
    w = slot.get();
  }
  std::lock_guard<std::mutex> lock(w->mu);
  if (w->bytes < need) {
    cudaError_t e = cudaSuccess;
    if (w->ptr != nullptr) {
      e = cudaStreamSynchronize(stream);
      if (e == cudaSuccess) e = cudaFree(w->ptr);
      w->ptr = nullptr;
      w->bytes = 0;
      if (e != cudaSuccess) return set_error(FA_ERR_CUDA, "workspace release: %s", cudaGetErrorString(e));
    }
    e = cudaMalloc(&w->ptr, need);
    if (e != cudaSuccess) {
      w->ptr = nullptr;
      return set_error(FA_ERR_CUDA, "workspace allocation (%zu bytes): %s", need,
                       cudaGetErrorString(e));
    }
    w->bytes = need;
  }
  *out = w->ptr;
  return FA_OK;
}

int ensure_device(int dev, DeviceState** out) {
  if (dev < 0 || dev >= kMaxDevices) return set_error(FA_ERR_CUDA, "device index %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_mutex);
  DeviceState& d = g_dev[dev];
  if (!d.ready) {
    if (g_encode == nullptr) {
      void* fn = nullptr;
      cudaDriverEntryPointQueryResult q;
      cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
      if (e != cudaSuccess || fn == nullptr || q != cudaDriverEntryPointSuccess)
        return set_error(FA_ERR_CUDA, "cuTensorMapEncodeTiled unavailable: %s",
                         cudaGetErrorString(e));
      g_encode = reinterpret_cast<EncodeTiledFn>(fn);
    }
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    if (major != 10 || minor != 0)
      return set_error(FA_ERR_UNSUPPORTED, "device %d is sm_%d%d; this kernel needs sm_100", dev,
                       major, minor);
    cudaError_t e = cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return set_error(FA_ERR_CUDA, "%s", cudaGetErrorString(e));
    for (const void* fn : {reinterpret_cast<const void*>(&fa::fa_fwd_kernel<false, true, false>),
                           reinterpret_cast<const void*>(&fa::fa_fwd_kernel<false, false, false>),
                           reinterpret_cast<const void*>(&fa::fa_fwd_kernel<true, false, false>),
                           reinterpret_cast<const void*>(&fa::fa_fwd_kernel<false, false, true>),
                           reinterpret_cast<const void*>(&fa::fa_fwd_kernel<false, true, false, true>),
                           reinterpret_cast<const void*>(&fa::fa_fwd_kernel<false, false, false, true>),
                           reinterpret_cast<const void*>(&fa::fa_fwd_kernel<true, false, false, true>),
                           reinterpret_cast<const void*>(&fa::fa_fwd_kernel<false, false, true, true>)}) {
      e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(fa::kSmemBytes));
      if (e != cudaSuccess) break;
    }
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(reinterpret_cast<const void*>(&fa::bwd::bwd_kernel),
                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(fa::bwd::kSmBytes));
    if (e != cudaSuccess)
      return set_error(FA_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    void* sym = nullptr;
    e = cudaGetSymbolAddress(&sym, fa::g_status_word);
    if (e != cudaSuccess)
      return set_error(FA_ERR_CUDA, "cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    d.status = static_cast<unsigned int*>(sym);
    // In host code g_noalloc_scratch names a host-side shadow, not device
    // memory: the device address is looked up here, once per device, with
    // that device current.
    void* scratch = nullptr;
    e = cudaGetSymbolAddress(&scratch, fa::g_noalloc_scratch);
    if (e != cudaSuccess)
      return set_error(FA_ERR_CUDA, "cudaGetSymbolAddress (scratch): %s", cudaGetErrorString(e));
    d.noalloc_scratch = scratch;
    d.ready = true;
  }
  *out = &d;
  return FA_OK;
}

// cuTensorMapEncodeTiled is a pure function of its arguments, so a small
// per-thread cache of recent maps is always valid; it saves the encoding when
// a caller reuses its buffers (a serving or benchmark loop), which matters for
// short problems whose kernel takes a few microseconds.
struct MapCacheEntry {
  CUtensorMap map;
  const void* ptr = nullptr;
  int64_t rows = -1, slices = -1;
  uint32_t box_rows = 0;
};
constexpr int kMapCacheSize = 8;
thread_local MapCacheEntry t_map_cache[kMapCacheSize];
thread_local int t_map_next = 0;

int make_map(CUtensorMap* map, const void* ptr, int64_t rows, int64_t slices,
             uint32_t box_rows) {
  for (const MapCacheEntry& e : t_map_cache) {
    if (e.ptr == ptr && e.rows == rows && e.slices == slices && e.box_rows == box_rows) {
      *map = e.map;
      return FA_OK;
    }
  }
  const cuuint64_t dims[3] = {64, static_cast<cuuint64_t>(rows), static_cast<cuuint64_t>(slices)};
  const cuuint64_t strides[2] = {128, static_cast<cuuint64_t>(rows) * 128};
  const cuuint32_t box[3] = {64, box_rows, 1};
  const cuuint32_t estride[3] = {1, 1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(ptr), dims,
                        strides, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(FA_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  MapCacheEntry& slot = t_map_cache[t_map_next];
  t_map_next = (t_map_next + 1) % kMapCacheSize;
  slot.map = *map;
  slot.ptr = ptr;
  slot.rows = rows;
  slot.slices = slices;
  slot.box_rows = box_rows;
  return FA_OK;
}

int launch(const void* q, const void* k, const void* v, void* o, int64_t bh, int64_t n_q,
           int64_t n_k, int causal, float scale, cudaStream_t stream, float* dbg,
           bool noalloc = false, float* lse = nullptr) {
  if (bh < 0 || n_q < 0 || n_k < 0) return set_error(FA_ERR_INVALID, "negative size");
  if (bh == 0 || n_q == 0) return FA_OK;
  if (n_k == 0) return set_error(FA_ERR_INVALID, "key length must be positive when queries exist");
  if (q == nullptr || k == nullptr || v == nullptr || o == nullptr)
    return set_error(FA_ERR_INVALID, "null pointer");
  const uintptr_t mis = reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
                        reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(o);
  if (mis & 15) return set_error(FA_ERR_INVALID, "q, k, v and o must be 16-byte aligned");
  if (n_q > (1ll << 30) || n_k > (1ll << 30) || bh > (1ll << 30))
    return set_error(FA_ERR_INVALID, "size too large");
  if (!(scale > 0.f) || !std::isfinite(scale)) return set_error(FA_ERR_INVALID, "scale must be positive and finite");
  const int64_t n_qpairs = ((n_q + 127) / 128 + 1) / 2;
  if (bh * n_qpairs > 0x7fffffffll) return set_error(FA_ERR_INVALID, "too many work items");

  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(FA_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  DeviceState* d = nullptr;
  int rc = ensure_device(dev, &d);
  if (rc != FA_OK) return rc;

  CUtensorMap tq, tk, tv, to;
  // q, k, v: 128-row tiles; o: 32-row slices (one TMA store per softmax warp)
  if ((rc = make_map(&tq, q, n_q, bh, 128)) != FA_OK) return rc;
  if ((rc = make_map(&tk, k, n_k, bh, 128)) != FA_OK) return rc;
  if ((rc = make_map(&tv, v, n_k, bh, 128)) != FA_OK) return rc;
  if ((rc = make_map(&to, o, n_q, bh, 32)) != FA_OK) return rc;

  fa::FwdParams p;
  p.n_q = static_cast<int>(n_q);
  p.n_k = static_cast<int>(n_k);
  p.bh = static_cast<int>(bh);
  p.causal = causal ? 1 : 0;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.n_qpairs = static_cast<int>(n_qpairs);
  p.n_items = static_cast<int>(bh * n_qpairs);
  p.status = d->status;
  p.limit_ns = g_wait_limit_ns.load(std::memory_order_relaxed);
  p.dbg = dbg;
  p.lse = lse;
  p.scale = scale;

  p.out = static_cast<__half*>(o);
  const SplitPlan sp = plan_split(bh, n_q, n_k, d->sms);
  p.n_split = sp.n_split;
  p.kv_chunk = sp.kv_chunk;
  p.n_qtiles = sp.n_qtiles;
  p.part_o = nullptr;
  p.part_ml = nullptr;
  p.counters = nullptr;
  if (sp.n_split > 1) {
    void* ws = nullptr;
    if (noalloc) {
      if (sp.total() > fa::kNoAllocScratchBytes)
        return set_error(FA_ERR_INVALID,
                         "this problem needs %zu bytes of scratch; fa_fwd_sm100_noalloc holds "
                         "at most %zu",
                         sp.total(), static_cast<size_t>(fa::kNoAllocScratchBytes));
      ws = d->noalloc_scratch;
    } else if ((rc = get_workspace(dev, stream, sp.total(), &ws)) != FA_OK) {
      return rc;
    }
    // The split counters must start at zero.  A completed launch leaves them
    // at zero, but one whose waits timed out can leave some set, so they are
    // cleared before every split launch (4 KiB, ordered on the stream).
    e = cudaMemsetAsync(ws, 0, sp.counters_bytes, stream);
    if (e != cudaSuccess) return set_error(FA_ERR_CUDA, "scratch clear: %s", cudaGetErrorString(e));
    uint8_t* base = static_cast<uint8_t*>(ws);
    p.counters = reinterpret_cast<int*>(base);
    p.part_ml = reinterpret_cast<float2*>(base + sp.counters_bytes);
    p.part_o = reinterpret_cast<float*>(base + sp.counters_bytes + sp.ml_bytes);
    p.n_items *= sp.n_split;
  }

  // Short problems: when the query tiles fit in one wave, make every 128-row
  // query tile its own work item (twice the blocks of the pair items; with
  // FA_HALVES the tile's key range is split between the two warpgroups).
  p.single = 0;
  if (p.n_split == 1 && static_cast<int64_t>(bh) * sp.n_qtiles <= d->sms) {
    p.single = 1;
    p.n_qpairs = sp.n_qtiles;
    p.n_items = static_cast<int>(bh * sp.n_qtiles);
  }
  p.unit = (p.n_split == 1 && p.n_items > d->sms) ? 2 : 1;
  const int units = (p.n_items + p.unit - 1) / p.unit;
  const int grid = units < d->sms ? units : d->sms;
  constexpr int kThr = fa::kNumThreads;
  constexpr uint32_t kSm = fa::kSmemBytes;
  if (lse != nullptr) {
    // the same four variants, each also writing the row log-sum-exp
    if (p.n_split > 1)
      fa::fa_fwd_kernel<true, false, false, true><<<grid, kThr, kSm, stream>>>(tq, tk, tv, to, p);
    else if (p.single && FA_HALVES)
      fa::fa_fwd_kernel<false, false, true, true><<<grid, kThr, kSm, stream>>>(tq, tk, tv, to, p);
    else if (!p.single && sp.n_qtiles % 2 == 0)
      fa::fa_fwd_kernel<false, true, false, true><<<grid, kThr, kSm, stream>>>(tq, tk, tv, to, p);
    else
      fa::fa_fwd_kernel<false, false, false, true><<<grid, kThr, kSm, stream>>>(tq, tk, tv, to, p);
  } else if (p.n_split > 1) {
    fa::fa_fwd_kernel<true, false, false><<<grid, kThr, kSm, stream>>>(tq, tk, tv, to, p);
  } else if (p.single && FA_HALVES) {
    // one query tile per block, its key range shared by both softmax warpgroups
    fa::fa_fwd_kernel<false, false, true><<<grid, kThr, kSm, stream>>>(tq, tk, tv, to, p);
  } else if (!p.single && sp.n_qtiles % 2 == 0) {
    // every work item is a pair of query tiles, each with at least one key tile
    fa::fa_fwd_kernel<false, true, false><<<grid, kThr, kSm, stream>>>(tq, tk, tv, to, p);
  } else {
    fa::fa_fwd_kernel<false, false, false><<<grid, kThr, kSm, stream>>>(tq, tk, tv, to, p);
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(FA_ERR_CUDA, "kernel launch: %s", cudaGetErrorString(e));
  return FA_OK;
}

}  // namespace

extern "C" {

int fa_fwd_sm100(const void* q, const void* k, const void* v, void* o, int64_t batch,
                 int64_t heads, int64_t seq_len, int causal, float scale, void* cuda_stream) {
  if (batch < 0 || heads < 0) return set_error(FA_ERR_INVALID, "negative size");
  return launch(q, k, v, o, batch * heads, seq_len, seq_len, causal, scale,
                static_cast<cudaStream_t>(cuda_stream), nullptr);
}

int fa_fwd_sm100_varlen(const void* q, const void* k, const void* v, void* o, int64_t batch,
                        int64_t heads, int64_t q_len, int64_t kv_len, int causal, float scale,
                        void* cuda_stream) {
  if (batch < 0 || heads < 0) return set_error(FA_ERR_INVALID, "negative size");
  return launch(q, k, v, o, batch * heads, q_len, kv_len, causal, scale,
                static_cast<cudaStream_t>(cuda_stream), nullptr);
}

int fa_fwd_sm100_noalloc(const void* q, const void* k, const void* v, void* o, int64_t batch,
                         int64_t heads, int64_t q_len, int64_t kv_len, int causal, float scale,
                         void* cuda_stream) {
  if (batch < 0 || heads < 0) return set_error(FA_ERR_INVALID, "negative size");
  return launch(q, k, v, o, batch * heads, q_len, kv_len, causal, scale,
                static_cast<cudaStream_t>(cuda_stream), nullptr, /*noalloc=*/true);
}

int fa_fwd_sm100_lse(const void* q, const void* k, const void* v, void* o, float* lse,
                     int64_t batch, int64_t heads, int64_t q_len, int64_t kv_len, int causal,
                     float scale, void* cuda_stream) {
  if (batch < 0 || heads < 0) return set_error(FA_ERR_INVALID, "negative size");
  if (lse == nullptr && batch * heads * q_len > 0) return set_error(FA_ERR_INVALID, "null pointer");
  return launch(q, k, v, o, batch * heads, q_len, kv_len, causal, scale,
                static_cast<cudaStream_t>(cuda_stream), nullptr, false, lse);
}

int fa_bwd_sm100_varlen(const void* q, const void* k, const void* v, const void* o,
                        const void* d_o, const float* lse, void* dq, void* dk, void* dv,
                        int64_t batch, int64_t heads, int64_t q_len, int64_t kv_len, int causal,
                        float scale, void* cuda_stream) {
  if (batch < 0 || heads < 0 || q_len < 0 || kv_len < 0)
    return set_error(FA_ERR_INVALID, "negative size");
  const int64_t bh = batch * heads, nq = q_len, nk = kv_len;
  if (bh == 0 || (nq == 0 && nk == 0)) return FA_OK;
  const void* ptrs[] = {q, k, v, o, d_o, lse, dq, dk, dv};
  for (const void* ptr : ptrs) {
    if (ptr == nullptr) return set_error(FA_ERR_INVALID, "null pointer");
    if (reinterpret_cast<uintptr_t>(ptr) & 15)
      return set_error(FA_ERR_INVALID, "tensors must be 16-byte aligned");
  }
  if (nq > (1ll << 30) || nk > (1ll << 30) || bh > (1ll << 30))
    return set_error(FA_ERR_INVALID, "size too large");
  if (!(scale > 0.f) || !std::isfinite(scale))
    return set_error(FA_ERR_INVALID, "scale must be positive and finite");
  if (nk == 0) return set_error(FA_ERR_INVALID, "key length must be positive when queries exist");
  const int64_t n_qt = (nq + 127) / 128, nq_pad = n_qt * 128;
  // causal (top-left): key tiles past the last query tile are seen by no query
  const int64_t n_kt_all = (nk + 127) / 128, n_kt = causal ? std::min(n_kt_all, n_qt) : n_kt_all;
  if (bh * n_kt > 0x7fffffffll) return set_error(FA_ERR_INVALID, "too many blocks");
  cudaStream_t stream = static_cast<cudaStream_t>(cuda_stream);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(FA_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  DeviceState* d = nullptr;
  int rc = ensure_device(dev, &d);
  if (rc != FA_OK) return rc;
  if (nq == 0) {  // no queries: dK = dV = 0
    const size_t bytes = static_cast<size_t>(bh) * nk * 64 * sizeof(__half);
    if ((e = cudaMemsetAsync(dk, 0, bytes, stream)) != cudaSuccess ||
        (e = cudaMemsetAsync(dv, 0, bytes, stream)) != cudaSuccess)
      return set_error(FA_ERR_CUDA, "dK/dV clear: %s", cudaGetErrorString(e));
    return FA_OK;
  }

  // scratch: [counter prefix of the split mode, left alone][row terms][dQ accumulator]
  const size_t rowterm_bytes = align256(static_cast<size_t>(bh) * nq_pad * 2 * sizeof(float));
  const size_t dq_bytes = static_cast<size_t>(bh) * nq_pad * 64 * sizeof(float);
  void* ws = nullptr;
  if ((rc = get_workspace(dev, stream, kCounterBytes + rowterm_bytes + dq_bytes, &ws)) != FA_OK)
    return rc;
  uint8_t* wb = static_cast<uint8_t*>(ws) + kCounterBytes;
  float* rowterm = reinterpret_cast<float*>(wb);
  float* dq_acc = reinterpret_cast<float*>(wb + rowterm_bytes);
  e = cudaMemsetAsync(dq_acc, 0, dq_bytes, stream);
  if (e != cudaSuccess) return set_error(FA_ERR_CUDA, "dQ clear: %s", cudaGetErrorString(e));
  if (n_kt * 128 < nk) {  // dK = dV = 0 for the keys of those tiles
    const size_t pitch = static_cast<size_t>(nk) * 64 * sizeof(__half);
    const size_t skip = static_cast<size_t>(n_kt) * 128 * 64 * sizeof(__half);
    if ((e = cudaMemset2DAsync(static_cast<uint8_t*>(dk) + skip, pitch, 0, pitch - skip, bh,
                               stream)) != cudaSuccess ||
        (e = cudaMemset2DAsync(static_cast<uint8_t*>(dv) + skip, pitch, 0, pitch - skip, bh,
                               stream)) != cudaSuccess)
      return set_error(FA_ERR_CUDA, "dK/dV clear: %s", cudaGetErrorString(e));
  }

  const int64_t rows_pad = bh * nq_pad;
  fa::bwd::rowterm_kernel<<<static_cast<unsigned>((rows_pad + 255) / 256), 256, 0, stream>>>(
      static_cast<const __half*>(o), static_cast<const __half*>(d_o), lse, rowterm,
      static_cast<int>(nq), static_cast<int>(nq_pad), rows_pad);
  e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(FA_ERR_CUDA, "kernel launch: %s", cudaGetErrorString(e));

  CUtensorMap tq, tk, tv, tdo;
  if ((rc = make_map(&tq, q, nq, bh, 128)) != FA_OK) return rc;
  if ((rc = make_map(&tk, k, nk, bh, 128)) != FA_OK) return rc;
  if ((rc = make_map(&tv, v, nk, bh, 128)) != FA_OK) return rc;
  if ((rc = make_map(&tdo, d_o, nq, bh, 128)) != FA_OK) return rc;
  fa::bwd::Params bp;
  bp.n_q = static_cast<int>(nq);
  bp.n_k = static_cast<int>(nk);
  bp.nq_pad = static_cast<int>(nq_pad);
  bp.bh = static_cast<int>(bh);
  bp.causal = causal ? 1 : 0;
  bp.n_kt = static_cast<int>(n_kt);
  bp.n_qt = static_cast<int>(n_qt);
  bp.scale = scale;
  bp.scale_log2 = scale * 1.4426950408889634f;
  bp.rowterm = rowterm;
  bp.dq_acc = dq_acc;
  bp.dk = static_cast<__half*>(dk);
  bp.dv = static_cast<__half*>(dv);
  bp.status = d->status;
  bp.limit_ns = g_wait_limit_ns.load(std::memory_order_relaxed);
  fa::bwd::bwd_kernel<<<static_cast<unsigned>(bh * n_kt), fa::bwd::kThreads, fa::bwd::kSmBytes,
                        stream>>>(tq, tk, tv, tdo, bp);
  e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(FA_ERR_CUDA, "kernel launch: %s", cudaGetErrorString(e));

  const int64_t rows = bh * nq;
  fa::bwd::dq_convert_kernel<<<static_cast<unsigned>((rows * 8 + 255) / 256), 256, 0, stream>>>(
      dq_acc, static_cast<__half*>(dq), static_cast<int>(nq), static_cast<int>(nq_pad), rows,
      scale);
  e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(FA_ERR_CUDA, "kernel launch: %s", cudaGetErrorString(e));
  return FA_OK;
}

int fa_bwd_sm100(const void* q, const void* k, const void* v, const void* o, const void* d_o,
                 const float* lse, void* dq, void* dk, void* dv, int64_t batch, int64_t heads,
                 int64_t seq_len, int causal, float scale, void* cuda_stream) {
  return fa_bwd_sm100_varlen(q, k, v, o, d_o, lse, dq, dk, dv, batch, heads, seq_len, seq_len,
                             causal, scale, cuda_stream);
}

int fa_fwd_sm100_debug(const void* q, const void* k, const void* v, void* o, int64_t batch,
                       int64_t heads, int64_t seq_len, int causal, float scale, void* cuda_stream,
                       float* score_dump) {
  return launch(q, k, v, o, batch * heads, seq_len, seq_len, causal, scale,
                static_cast<cudaStream_t>(cuda_stream), score_dump);
}

const char* fa_last_error(void) { return g_last_error; }

int fa_read_status(void* cuda_stream, unsigned int* status_out, int clear) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(FA_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  DeviceState* d = nullptr;
  int rc = ensure_device(dev, &d);
  if (rc != FA_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(cuda_stream);
  unsigned int v = 0;
  e = cudaMemcpyAsync(&v, d->status, sizeof(v), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return set_error(FA_ERR_CUDA, "status read: %s", cudaGetErrorString(e));
  if (clear) {
    e = cudaMemsetAsync(d->status, 0, sizeof(unsigned int), s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return set_error(FA_ERR_CUDA, "status clear: %s", cudaGetErrorString(e));
  }
  if (status_out) *status_out = v;
  return FA_OK;
}

void fa_set_wait_limit_ns(unsigned long long limit_ns) {
  g_wait_limit_ns.store(limit_ns == 0 ? kDefaultWaitLimitNs : limit_ns, std::memory_order_relaxed);
}

int fa_selftest_wait_timeout(unsigned long long limit_ns, void* cuda_stream) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(FA_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  DeviceState* d = nullptr;
  int rc = ensure_device(dev, &d);
  if (rc != FA_OK) return rc;
  fa::selftest_timeout_kernel<<<1, 32, 0, static_cast<cudaStream_t>(cuda_stream)>>>(d->status,
                                                                                  limit_ns);
  e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(FA_ERR_CUDA, "kernel launch: %s", cudaGetErrorString(e));
  return FA_OK;
}

int fa_smem_bytes(void) { return static_cast<int>(fa::kSmemBytes); }

void fa_set_max_splits(int max_splits) {
  g_max_splits.store(max_splits < 0 ? 0 : max_splits, std::memory_order_relaxed);
}

int fa_release_workspaces(void) {
  std::lock_guard<std::mutex> lock(g_mutex);
  int prev = 0;
  cudaGetDevice(&prev);
  int rc = FA_OK;
  for (auto& kv : g_workspaces) {
    Workspace& w = *kv.second;
    std::lock_guard<std::mutex> wl(w.mu);
    if (w.ptr == nullptr) continue;
    cudaError_t e = cudaSetDevice(kv.first.first);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaFree(w.ptr);
    if (e != cudaSuccess) rc = set_error(FA_ERR_CUDA, "workspace release: %s", cudaGetErrorString(e));
    w.ptr = nullptr;
    w.bytes = 0;
  }
  g_workspaces.clear();
  cudaSetDevice(prev);
  return rc;
}

}  // extern "C"
