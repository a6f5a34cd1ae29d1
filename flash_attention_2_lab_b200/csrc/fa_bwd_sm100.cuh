// Attention backward for B200 (sm_100a), head dimension 64, fp16 inputs and
// gradients, fp32 accumulation.  Included by fa_fwd_sm100.cu (it shares the
// PTX wrappers, the status word and the host plumbing there).
//
// Not in the reference (its kernels are forward only); this is the training
// half of the same attention: given Q, K, V, O, dO and the forward's row
// log-sum-exp L,
//   P  = exp(scale * Q K^T - L)          (recomputed, causal mask applied)
//   dV = P^T dO,   dP = dO V^T,   dS = P * (dP - D),   D = rowsum(dO * O)
//   dK = scale * dS^T Q,          dQ = scale * dS K
//
// Query length n_q and key length n_k may differ (causal mask top-left: key
// k is seen by queries q >= k, as in the forward).  One block per
// (batch*head, 128-key tile j), head-major; it keeps K_j, V_j, dK_j and dV_j
// on chip and walks the query tiles i (all of them, or i >= j when causal;
// key tiles that no query reaches get no block, the host clears their dK,
// dV):
//
//   warp 8   TMA producer: K_j, V_j once; per query tile Q_i, dO_i and the
//            row terms (L * log2 e, D) into a two-slot ring.
//   warp 10  issues one bulk asynchronous reduction per query tile (dQ_i
//            staging -> global fp32 accumulator) and frees the staging buffer
//            once the reduction has read it, off the compute warps' path.
//   warp 9   MMA issuer and TMEM owner.  Per query tile:
//              S^T  = K_j Q_i^T   (SS, 128 keys x 128 queries)     -> TMEM
//              dP^T = V_j dO_i^T  (SS)                              -> TMEM
//            then S^T of tile i+1 as soon as the exponentials of tile i
//            have read S^T, and once the compute warps have written P^T and
//            dS^T (the exponentials of tile i+1 overlap these three):
//              dV  += P^T  dO_i   (TS, P^T read from TMEM)
//              dK  += dS^T Q_i    (TS, dS^T read from TMEM)
//              dQ_i = dS K_j      (SS; dS^T staged in shared memory is read
//                                  as an MN-major A operand) -> dP^T columns
//            and dP^T of tile i+1 once dQ_i has been read.
//   warps 0-7  compute, two warps per TMEM lane quadrant (warp w and w + 4
//            take query columns 0-63 and 64-127 of the same rows): for key
//            row k, p = 2^(s c - L log2 e) (kept in registers as fp16 until
//            the previous tile's dV MMA is done), ds = p (dp - D) with that
//            fp16 p, both into TMEM (and ds into shared memory).
//   warps 11-14 dQ_i readout, one warp per TMEM lane quadrant (lane = query
//            row): the fp32 dQ_i tile goes to a staging buffer in shared
//            memory, from which one bulk asynchronous reduction (TMA unit,
//            issued by warp 10) adds it into the global fp32 dQ accumulator
//            (32 KiB, contiguous: the other key tiles add theirs; the 16-byte
//            chunks of each half-row sit XOR-swizzled by the row, which
//            dq_convert_kernel undoes).
//
// Tensor memory (512 columns): S^T 0-127, dP^T 128-255 (dQ_i reuses 128-191
// once dP^T is consumed), P^T 256-319 (fp16 pairs), dS^T 320-383 (fp16
// pairs), dV 384-447, dK 448-511.
//
// Shared-memory descriptors of MN-major operands (128-byte swizzle): an atom
// is 8 rows of the K dimension x 64 fp16 of the MN dimension (128 B per
// row); the leading byte offset is the stride between atoms along MN and the
// stride byte offset the stride between 8-row groups along K.
//
// Every wait is bounded, as in the forward kernel.
#pragma once

#include <type_traits>

namespace fa {
namespace bwd {

constexpr int kThreads = 480;
constexpr int kQSlots = 2;
constexpr int kComputeWarps = 8;
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kReduceWarp = 10;  // issues the bulk dQ reductions
constexpr int kDqWarp0 = 11;     // warps 11-14 read and stage dQ_i, one per TMEM lane quadrant
constexpr int kDqWarps = 4;

constexpr uint32_t kSmK = 0;
constexpr uint32_t kSmV = kSmK + kTileBytes;
constexpr uint32_t kSmQ = kSmV + kTileBytes;
constexpr uint32_t kSmDO = kSmQ + kQSlots * kTileBytes;
constexpr uint32_t kSmDS = kSmDO + kQSlots * kTileBytes;  // two 64-query halves, 16 KiB each
constexpr uint32_t kSmVec = kSmDS + 2 * kTileBytes;       // per slot: 128 L log2 e, 128 D
constexpr uint32_t kVecBytes = 128 * 2 * sizeof(float);
constexpr uint32_t kSmDQ = kSmVec + kQSlots * kVecBytes;  // fp32 dQ_i staging, 128 x 64
constexpr uint32_t kDQBytes = 128 * 64 * sizeof(float);
constexpr uint32_t kSmCtl = kSmDQ + kDQBytes;
constexpr uint32_t kSmBytes = kSmCtl + 256 + 1024;  // + alignment slack

constexpr uint32_t kColS = 0, kColDP = 128, kColP = 256, kColDS = 320, kColDV = 384,
                   kColDK = 448;

struct Ctl {
  uint64_t kv_full;
  uint64_t q_full[kQSlots], q_empty[kQSlots];
  uint64_t s_full, s_free, dp_full, p_full, dq_full, dq_free;
  uint64_t dqs_full, dqs_free;  // dQ staging written by the 4 dQ warps / read by the reduction
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};
static_assert(sizeof(Ctl) <= 256, "control block too large");

struct Params {
  int n_q;           // query rows per (batch, head)
  int n_k;           // key rows per (batch, head)
  int nq_pad;        // n_q rounded up to 128 (rows of the row-term and dQ buffers)
  int bh;
  int causal;        // top-left: key k is seen by queries q >= k
  int n_kt;          // key tiles with at least one query per (batch, head): one block each
  int n_qt;          // query tiles per (batch, head)
  float scale;       // softmax scale
  float scale_log2;  // scale * log2(e)
  const float* rowterm;   // [bh][nq_pad / 128][2][128]: per query tile L log2 e, then D
  float* dq_acc;          // [bh][nq_pad][64] fp32, zeroed before the launch
  __half* dk;             // [bh][n_k][64]
  __half* dv;
  unsigned int* status;
  unsigned long long limit_ns;
};

__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes,
                                          uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(dst),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(bar)
      : "memory");
}

// global[dst .. dst + bytes) += shared[src ..), fp32, by the TMA unit
__device__ __forceinline__ void bulk_reduce_add_f32(float* dst, uint32_t src, uint32_t bytes) {
  asm volatile("cp.reduce.async.bulk.global.shared::cta.bulk_group.add.f32 [%0], [%1], %2;" ::"l"(
                   reinterpret_cast<uint64_t>(dst)),
               "r"(src), "r"(bytes)
               : "memory");
}

// First query tile of key tile j (top-left causal mask: key k is seen by
// queries q >= k, i.e. query tiles i >= j).
__device__ __forceinline__ int first_qtile(const Params& p, int j) { return p.causal ? j : 0; }

__global__ void __launch_bounds__(kThreads, 1)
    bwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
               const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
               const Params p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;  // SW128 tiles need 1 KiB alignment
  uint8_t* gen_base = smem_raw + (base - raw);
  Ctl* ctl = reinterpret_cast<Ctl*>(gen_base + kSmCtl);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  // head-major: the key-tile blocks of one head run together and share its Q,
  // dO and dQ tiles in L2
  const int bh = blockIdx.x / p.n_kt;
  const int j = blockIdx.x % p.n_kt;
  const int i0 = first_qtile(p, j);
  const int n_steps = p.n_qt - i0;
  volatile int* abort_flag = &ctl->abort;
  auto qtile = [&](int it) { return i0 + it; };

  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&ctl->kv_full), 1);
    for (int s = 0; s < kQSlots; ++s) {
      mbar_init(smem_u32(&ctl->q_full[s]), 1);
      mbar_init(smem_u32(&ctl->q_empty[s]), 1);
    }
    mbar_init(smem_u32(&ctl->s_full), 1);
    mbar_init(smem_u32(&ctl->dp_full), 1);
    mbar_init(smem_u32(&ctl->s_free), kComputeWarps);
    mbar_init(smem_u32(&ctl->p_full), kComputeWarps);
    mbar_init(smem_u32(&ctl->dq_full), 1);
    mbar_init(smem_u32(&ctl->dq_free), kDqWarps);
    mbar_init(smem_u32(&ctl->dqs_full), kDqWarps);
    mbar_init(smem_u32(&ctl->dqs_free), 1);
    mbar_init(smem_u32(&ctl->drain), 1);
    ctl->abort = 0;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(smem_u32(&ctl->tmem_base), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;

  if (warp == kProducerWarp) {
    // ------------------------------------------------------------ producer
    if (elect_one()) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      tma_prefetch_desc(&tm_do);
      const uint32_t kv = smem_u32(&ctl->kv_full);
      mbar_arrive_expect_tx(kv, 2 * kTileBytes);
      tma_load_3d(base + kSmK, &tm_k, kv, 0, j * 128, bh);
      tma_load_3d(base + kSmV, &tm_v, kv, 0, j * 128, bh);
    }
    __syncwarp();
    int issued = 0;
    for (int it = 0; it < n_steps; ++it) {
      const int i = i0 + it, slot = it % kQSlots;
      if (!mbar_wait_warp(smem_u32(&ctl->q_empty[slot]), ((it / kQSlots) & 1) ^ 1, abort_flag,
                          p.status, kStatusTimeoutProducer, p.limit_ns))
        break;
      if (elect_one()) {
        const uint32_t full = smem_u32(&ctl->q_full[slot]);
        mbar_arrive_expect_tx(full, 2 * kTileBytes + kVecBytes);
        tma_load_3d(base + kSmQ + slot * kTileBytes, &tm_q, full, 0, i * 128, bh);
        tma_load_3d(base + kSmDO + slot * kTileBytes, &tm_do, full, 0, i * 128, bh);
        bulk_load(base + kSmVec + slot * kVecBytes,
                  p.rowterm + (static_cast<size_t>(bh) * p.nq_pad + i * 128) * 2, kVecBytes, full);
      }
      __syncwarp();
      issued = it + 1;
    }
    // Let every copy started land before the block exits (bounded).
    if (lane == 0) {
      mbar_wait(smem_u32(&ctl->kv_full), 0, nullptr, p.status, kStatusTimeoutDrain,
                kDrainLimitNs);
      for (int it = issued - 1; it >= 0 && it >= issued - kQSlots; --it)
        mbar_wait(smem_u32(&ctl->q_full[it % kQSlots]), (it / kQSlots) & 1, nullptr, p.status,
                  kStatusTimeoutDrain, kDrainLimitNs);
    }
    __syncwarp();
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issuer
    constexpr uint32_t idesc_s = idesc_f16_f32(128, 128, false);
    constexpr uint32_t idesc_g = idesc_f16_f32(128, 64, true);  // B (dO, Q) MN-major
    // dQ = dS K: A = dS read MN-major (queries contiguous), B = K MN-major.
    constexpr uint32_t idesc_dq = idesc_f16_f32(128, 64, true) | (1u << 15);
    const uint64_t dk_ = smem_desc_sw128(base + kSmK, 16, 1024);
    const uint64_t dv_ = smem_desc_sw128(base + kSmV, 16, 1024);
    const uint64_t dds = smem_desc_sw128(base + kSmDS, kTileBytes, 1024);
    constexpr uint64_t kTileDesc = kTileBytes >> 4;
    auto wait = [&](uint32_t bar, uint32_t parity) {
      return mbar_wait_warp(bar, parity, abort_flag, p.status, kStatusTimeoutMma, p.limit_ns);
    };
    const uint64_t dq0 = smem_desc_sw128(base + kSmQ, 16, 1024);
    const uint64_t ddo0 = smem_desc_sw128(base + kSmDO, 16, 1024);
    auto issue_s = [&](int it) {  // S^T = K_j Q_i^T
      const uint64_t dq_ = dq0 + (it % kQSlots) * kTileDesc;
      if (elect_one()) {
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_ss_f16(tmem + kColS, dk_ + 2 * kk, dq_ + 2 * kk, idesc_s, kk > 0);
        tc_commit(smem_u32(&ctl->s_full));
      }
      __syncwarp();
    };
    auto issue_dp = [&](int it) {  // dP^T = V_j dO_i^T
      const uint64_t ddo = ddo0 + (it % kQSlots) * kTileDesc;
      if (elect_one()) {
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_ss_f16(tmem + kColDP, dv_ + 2 * kk, ddo + 2 * kk, idesc_s, kk > 0);
        tc_commit(smem_u32(&ctl->dp_full));
      }
      __syncwarp();
    };
    bool ok = wait(smem_u32(&ctl->kv_full), 0) && n_steps > 0 && wait(smem_u32(&ctl->q_full[0]), 0);
    if (ok) {
      tc_fence_after();
      issue_s(0);
      issue_dp(0);
    }
    for (int it = 0; ok && it < n_steps; ++it) {
      const int slot = it % kQSlots;
      if (it + 1 < n_steps) {
        // S^T of the next tile once this tile's exponentials have read S^T
        if (!wait(smem_u32(&ctl->s_free), it & 1)) break;
        if (!wait(smem_u32(&ctl->q_full[(it + 1) % kQSlots]), ((it + 1) / kQSlots) & 1)) break;
        tc_fence_after();
        issue_s(it + 1);
      }
      // P^T, dS^T written; dP^T of this tile read
      if (!wait(smem_u32(&ctl->p_full), it & 1)) break;
      tc_fence_after();
      const uint64_t dq_ = dq0 + slot * kTileDesc;
      const uint64_t ddo = ddo0 + slot * kTileDesc;
      if (elect_one()) {
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)  // 16 queries per step
          mma_ts_f16(tmem + kColDV, tmem + kColP + kk * 8, ddo + 128 * kk, idesc_g,
                     (it > 0 || kk > 0) ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          mma_ts_f16(tmem + kColDK, tmem + kColDS + kk * 8, dq_ + 128 * kk, idesc_g,
                     (it > 0 || kk > 0) ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)  // 16 keys per step
          mma_ss_f16(tmem + kColDP, dds + 128 * kk, dk_ + 128 * kk, idesc_dq, kk > 0);
        tc_commit(smem_u32(&ctl->dq_full));
        tc_commit(smem_u32(&ctl->q_empty[slot]));
      }
      __syncwarp();
      if (it + 1 < n_steps) {
        // dP^T of the next tile goes over dQ_i: wait until it has been read
        if (!wait(smem_u32(&ctl->dq_free), it & 1)) break;
        tc_fence_after();
        issue_dp(it + 1);
      }
    }
    if (lane == 0) {
      tc_commit(smem_u32(&ctl->drain));
      mbar_wait(smem_u32(&ctl->drain), 0, nullptr, p.status, kStatusTimeoutDrain, kDrainLimitNs);
    }
    __syncwarp();
  } else if (warp == kReduceWarp) {
    // ------------------------------------------------------------ dQ reductions
    for (int it = 0; it < n_steps; ++it) {
      if (!mbar_wait_warp(smem_u32(&ctl->dqs_full), it & 1, abort_flag, p.status,
                          kStatusTimeoutSoftmax, p.limit_ns))
        break;
      if (lane == 0) {
        bulk_reduce_add_f32(p.dq_acc + (static_cast<size_t>(bh) * p.nq_pad + qtile(it) * 128) * 64,
                            base + kSmDQ, kDQBytes);
        bulk_commit_group();
        bulk_wait_group_read0();  // the staging buffer has been read
        mbar_arrive(smem_u32(&ctl->dqs_free));
      }
      __syncwarp();
    }
    // every reduction lands before the block exits
    if (lane == 0) bulk_wait_group0();
    __syncwarp();
  } else if (warp >= kDqWarp0) {
    // ------------------------------------------------------------ dQ_i readout
    // lane = query row of the tile; each warp reads its lane quadrant's 64
    // fp32 dQ columns and stages them for the reduction
    const int quad = warp % 4;
    const int r = quad * 32 + lane;
    const uint32_t t_dq = tmem + (static_cast<uint32_t>(quad * 32) << 16) + kColDP;
    auto wait = [&](uint32_t bar, uint32_t parity) {
      return mbar_wait_warp(bar, parity, abort_flag, p.status, kStatusTimeoutSoftmax,
                            p.limit_ns);
    };
    for (int it = 0; it < n_steps; ++it) {
      if (!wait(smem_u32(&ctl->dq_full), it & 1)) break;
      tc_fence_after();
      uint32_t dq[2][32];
      tmem_ld32(t_dq, dq[0]);
      tmem_ld32(t_dq + 32, dq[1]);
      tc_wait_ld32(dq[0]);
      tc_wait_ld32(dq[1]);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&ctl->dq_free));  // TMEM columns free for dP^T
      // the staging buffer is rewritten once the previous reduction has read it
      if (it > 0 && !wait(smem_u32(&ctl->dqs_free), (it - 1) & 1)) break;
      // row r: 64 floats = 16 chunks of 16 B in two halves; chunk c of a half
      // sits at position c ^ (r & 7) of that half (the accumulator keeps that
      // order; eight consecutive rows hit eight different bank groups)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t srow = base + kSmDQ + r * 256 + h * 128;
#pragma unroll
        for (int e = 0; e < 8; ++e)
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(srow + ((e ^ (r & 7)) << 4)),
                       "r"(dq[h][4 * e]), "r"(dq[h][4 * e + 1]), "r"(dq[h][4 * e + 2]),
                       "r"(dq[h][4 * e + 3])
                       : "memory");
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&ctl->dqs_full));
    }
  } else {
    // ------------------------------------------------------------ compute
    const int quad = warp % 4, half = warp / 4;  // lane quadrant, query-column half
    const int r = quad * 32 + lane;  // TMEM lane: key row, then query row of dQ
    const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t t_s = tmem + lane_base + kColS, t_dp = tmem + lane_base + kColDP;
    const uint32_t t_p = tmem + lane_base + kColP, t_ds = tmem + lane_base + kColDS;
    const int key = j * 128 + r;
    const float c = p.scale_log2;
    auto wait = [&](uint32_t bar, uint32_t parity) {
      return mbar_wait_warp(bar, parity, abort_flag, p.status, kStatusTimeoutSoftmax,
                            p.limit_ns);
    };
    // keys past n and (causal) queries before this key contribute nothing
    const int q_lo = p.causal ? key : 0;  // first query that sees this key
    const bool key_ok = key < p.n_k;
    const int key_max = j * 128 + quad * 32 + 31;  // last key of this warp
    // p of this warp's 64 queries of tile it, fp16 pairs: pk[16 c + u / 2]
    // holds queries 32 (2 half + c) + u, + 1
    uint32_t pk[32];
    // exponentials of tile it from S^T (needs S^T and the row terms of tile it)
    auto phase_p = [&](int it) -> bool {
      const int i = i0 + it, slot = it % kQSlots;
      if (!wait(smem_u32(&ctl->q_full[slot]), (it / kQSlots) & 1)) return false;
      if (!wait(smem_u32(&ctl->s_full), it & 1)) return false;
      tc_fence_after();
      const float* l2 = reinterpret_cast<const float*>(gen_base + kSmVec + slot * kVecBytes);
      // masks only where this warp's 32 keys x 64 queries reach past n or
      // (causal) below the diagonal
      const int q_min = i * 128 + 64 * half;
      const bool masked = key_max >= p.n_k || q_min + 63 >= p.n_q || (p.causal && q_min < key_max);
      auto exps = [&](auto mask_tag) {
        constexpr bool kMask = decltype(mask_tag)::value;
#pragma unroll
        for (int c2 = 0; c2 < 2; ++c2) {
          const int ch = 2 * half + c2;
          uint32_t sr[32];
          tmem_ld32(t_s + 32 * ch, sr);
          tc_wait_ld32(sr);
#pragma unroll
          for (int u = 0; u < 32; u += 4) {
            const int ql = 32 * ch + u;  // query within the tile
            const float4 lv = *reinterpret_cast<const float4*>(l2 + ql);
            const float lq[4] = {lv.x, lv.y, lv.z, lv.w};
            float pv[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              pv[e] = ex2_approx(__uint_as_float(sr[u + e]) * c - lq[e]);
              if (kMask) {
                const int q = i * 128 + ql + e;
                if (!key_ok || q < q_lo || q >= p.n_q) pv[e] = 0.f;
              }
            }
            pk[16 * c2 + u / 2] = pack_half2(pv[0], pv[1]);
            pk[16 * c2 + u / 2 + 1] = pack_half2(pv[2], pv[3]);
          }
        }
      };
      if (masked)
        exps(std::true_type{});
      else
        exps(std::false_type{});
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&ctl->s_free));  // S^T read: the next one may start
      return true;
    };
    bool ok = phase_p(0);
    for (int it = 0; ok && it < n_steps; ++it) {
      const int slot = it % kQSlots;
      // P^T of tile it into TMEM: the previous tile's dV MMA (which read the
      // columns) completed before its dQ was signalled
#pragma unroll
      for (int c2 = 0; c2 < 2; ++c2) tmem_st16(t_p + 16 * (2 * half + c2), pk + 16 * c2);
      if (!wait(smem_u32(&ctl->dp_full), it & 1)) { ok = false; break; }
      tc_fence_after();
      const float* dvec =
          reinterpret_cast<const float*>(gen_base + kSmVec + slot * kVecBytes) + 128;
#pragma unroll
      for (int c2 = 0; c2 < 2; ++c2) {
        const int ch = 2 * half + c2;
        uint32_t dpr[32];
        tmem_ld32(t_dp + 32 * ch, dpr);
        tc_wait_ld32(dpr);
        uint32_t dk16[16];
#pragma unroll
        for (int u = 0; u < 32; u += 4) {
          const float4 dv4 = *reinterpret_cast<const float4*>(dvec + 32 * ch + u);  // D
          const float2 pa = __half22float2(*reinterpret_cast<const __half2*>(&pk[16 * c2 + u / 2]));
          const float2 pb =
              __half22float2(*reinterpret_cast<const __half2*>(&pk[16 * c2 + u / 2 + 1]));
          dk16[u / 2] = pack_half2(pa.x * (__uint_as_float(dpr[u]) - dv4.x),
                                   pa.y * (__uint_as_float(dpr[u + 1]) - dv4.y));
          dk16[u / 2 + 1] = pack_half2(pb.x * (__uint_as_float(dpr[u + 2]) - dv4.z),
                                       pb.y * (__uint_as_float(dpr[u + 3]) - dv4.w));
        }
        tmem_st16(t_ds + 16 * ch, dk16);
        // dS^T row r, queries 32 ch .. 32 ch + 31: half ch / 2 of the staged
        // tile, four 16-byte chunks of its 128-byte row (128B swizzle)
        const uint32_t row_addr = base + kSmDS + (ch / 2) * kTileBytes + r * 128;
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          const int chunk = (ch % 2) * 4 + q4;
          const uint32_t dst = row_addr + ((chunk ^ (r & 7)) << 4);
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(dst), "r"(dk16[4 * q4]),
                       "r"(dk16[4 * q4 + 1]), "r"(dk16[4 * q4 + 2]), "r"(dk16[4 * q4 + 3])
                       : "memory");
        }
      }
      tc_wait_st();
      fence_proxy_async_smem();  // dS^T in shared memory is read by the MMA (async proxy)
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&ctl->p_full));
      // ---- exponentials of the next tile while the tensor cores run this one's
      // dV, dK, dQ
      if (it + 1 < n_steps && !phase_p(it + 1)) { ok = false; break; }
      // this tile's dV, dK, dQ MMAs have read P^T and dS^T (TMEM and shared
      // memory) before the next tile's are written
      if (!wait(smem_u32(&ctl->dq_full), it & 1)) { ok = false; break; }
    }
    // ---- dK_j, dV_j (lane = key row): after the last dQ_i signal, every MMA is done.
    // The TMEM loads are warp-collective: every lane takes part, only the
    // lanes of keys below n store.
    if (ok) {
      const size_t row = static_cast<size_t>(bh) * p.n_k + (key < p.n_k ? key : 0);
      {
        const int which = half;  // half 0 writes dV, half 1 dK
        const uint32_t col = which ? kColDK : kColDV;
        const float mul = which ? p.scale : 1.f;
        __half* out = (which ? p.dk : p.dv) + row * 64;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint32_t g[32];
          tmem_ld32(tmem + lane_base + col + 32 * h, g);
          tc_wait_ld32(g);
          uint32_t hv[16];
#pragma unroll
          for (int e = 0; e < 16; ++e)
            hv[e] = pack_half2(__uint_as_float(g[2 * e]) * mul, __uint_as_float(g[2 * e + 1]) * mul);
          uint4* o4 = reinterpret_cast<uint4*>(out + 32 * h);
          if (key < p.n_k) {
#pragma unroll
            for (int e = 0; e < 4; ++e)
              o4[e] = make_uint4(hv[4 * e], hv[4 * e + 1], hv[4 * e + 2], hv[4 * e + 3]);
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// Row terms for the backward: L log2 e and D = rowsum(dO * O) per query row,
// zero for the padding rows up to n_pad, stored per 128-query tile as 128 L
// values then 128 D values.  One thread per row.
__global__ void rowterm_kernel(const __half* __restrict__ o, const __half* __restrict__ d_o,
                               const float* __restrict__ lse, float* __restrict__ rowterm,
                               int n, int n_pad, int64_t rows_pad) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= rows_pad) return;
  const int64_t bh = idx / n_pad;
  const int q = static_cast<int>(idx - bh * n_pad);
  float l2 = 0.f, dsum = 0.f;
  if (q < n) {
    const size_t row = static_cast<size_t>(bh) * n + q;
    const uint4* a = reinterpret_cast<const uint4*>(o + row * 64);
    const uint4* b = reinterpret_cast<const uint4*>(d_o + row * 64);
    float acc = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const uint4 va = a[e], vb = b[e];
      const uint32_t wa[4] = {va.x, va.y, va.z, va.w}, wb[4] = {vb.x, vb.y, vb.z, vb.w};
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const float2 fa = __half22float2(*reinterpret_cast<const __half2*>(&wa[w]));
        const float2 fb = __half22float2(*reinterpret_cast<const __half2*>(&wb[w]));
        acc = fmaf(fa.x, fb.x, fmaf(fa.y, fb.y, acc));
      }
    }
    l2 = lse[row] * 1.4426950408889634f;
    dsum = acc;
  }
  // tile-blocked: 128 L log2 e, then 128 D, per query tile
  float* dst = rowterm + (idx - (q & 127)) * 2 + (q & 127);
  dst[0] = l2;
  dst[128] = dsum;
}

// dq = scale * dq_acc, fp32 -> fp16, rows below n.
__global__ void dq_convert_kernel(const float* __restrict__ dq_acc, __half* __restrict__ dq,
                                  int n, int n_pad, int64_t rows, float scale) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;  // (row, 8-col group)
  if (idx >= rows * 8) return;
  const int64_t row = idx / 8;
  const int g = static_cast<int>(idx % 8);
  const int64_t bh = row / n;
  const int q = static_cast<int>(row - bh * n);
  // chunk c (4 floats) of a 32-float half sits at position c ^ (q & 7)
  const float4* src = reinterpret_cast<const float4*>(dq_acc + (static_cast<size_t>(bh) * n_pad + q) * 64);
  const int c0 = 2 * g, hb = c0 & 8, sw = q & 7;
  const float4 a = src[hb | ((c0 & 7) ^ sw)], b = src[hb | (((c0 + 1) & 7) ^ sw)];
  uint4 out;
  out.x = pack_half2(a.x * scale, a.y * scale);
  out.y = pack_half2(a.z * scale, a.w * scale);
  out.z = pack_half2(b.x * scale, b.y * scale);
  out.w = pack_half2(b.z * scale, b.w * scale);
  reinterpret_cast<uint4*>(dq + row * 64)[g] = out;
}

}  // namespace bwd
}  // namespace fa
