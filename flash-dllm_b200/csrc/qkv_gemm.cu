// Fused QKV projection + RoPE + KV-cache scatter on tcgen05 tensor cores.
//
// Persistent kernel: one CTA per SM walks a list of work units; a unit is a
// 128-row x BN-column tile of [Q | K | V] = Xn * W^T for one projection and
// one head (BN = 128) or one half-head pair (BN = 64: columns c..c+31 and
// 64+c..64+c+31 of a head, so each RoPE pair stays in the tile), over one
// slice of K when the tile is split along K.  Warp roles (192 threads):
//   warp 0      TMA producer: X and W tiles (128-byte swizzle) into a deep
//               smem ring that runs on across units, completion on `full`
//               mbarriers (X boxes hold only the valid rows when <= 64);
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer into one
//               of two TMEM accumulators (units alternate), releasing ring
//               slots with tcgen05.commit on `empty`;
//   warps 2-5   epilogue of the previous unit while the next one accumulates:
//               TMEM -> registers (thread = row), split-K reduction, RoPE in
//               fp32 with the row's slot sin/cos, bf16 stores of Q to its row
//               and of K/V straight to cache[pos].
// Split units of one tile run on different CTAs at the same time; each writes
// its fp32 partial to the caller's workspace and the last to arrive (atomic
// counter) adds the others in split order, runs the epilogue and resets the
// counter for the next call.  (K splits only on request: whole-K tiles
// measured faster at every row count.)
//
// qkv2_rope_kernel (further down): the CTA-pair variant used for 129-256
// rows -- 2-SM UMMAs on 256 x 256 tiles, stream-K over (tile, k-block).
//
// Both kernels are launched programmatically dependent on the kernel before
// them (the RMSNorm producing X) and let the attention kernel after them
// launch early; they wait for X before their first load.
#include "common.cuh"
#include "internal.h"

namespace fdllm {

constexpr int kQkvBM = 128;
constexpr int kQkvBK = 64;
constexpr int kQkvThreads = 192;
constexpr int kQkvKernelId = 1;
constexpr int kQkvRingBytes = 192 * 1024;

// A ring slot holds KSUB 64-wide K sub-tiles of X and W (one 128-byte swizzle
// box per operand row each), i.e. 128 * KSUB contiguous bytes of every row.
template <int BN, int XROWS, int KSUB>
struct QkvCfg {
  static constexpr int kASub = XROWS * kQkvBK * 2;  // MMA reads 128 rows; rows >= XROWS are unused
  static constexpr int kBSub = BN * kQkvBK * 2;
  static constexpr int kABytes = KSUB * kASub;
  static constexpr int kBBytes = KSUB * kBSub;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = kQkvRingBytes / kStageBytes;
  static constexpr int kBarOffset = kStages * kStageBytes;
  static constexpr int kSmem = 1024 + kBarOffset + 256;
  static constexpr int kTmemCols = 2 * BN;  // two accumulators
};

struct QkvParams {
  const int64_t* pos;
  const float* sin;
  const float* cos;
  __nv_bfloat16* q_out;
  __nv_bfloat16* k_out;
  __nv_bfloat16* v_out;
  float* partials;
  int32_t* counters;
  int32_t* status;
  int64_t n_slots;
  int32_t n_rows;
  int32_t d_model;
  int32_t n_heads;
  int32_t kv_by_slot;
  int32_t splits;
  int32_t kb_per_split;
  int32_t m_tiles;
  int32_t n_units;
  int32_t ksub;
};

struct QkvUnit {
  int m_tile, n_tile, split, kb0, nkb;
};

__device__ __forceinline__ QkvUnit qkv_unit(const QkvParams& p, int u) {
  QkvUnit w;
  const int tile = u / p.splits;
  w.split = u % p.splits;
  w.m_tile = tile % p.m_tiles;
  w.n_tile = tile / p.m_tiles;
  const int kb_total = p.d_model / (kQkvBK * p.ksub);
  w.kb0 = w.split * p.kb_per_split;
  w.nkb = min(kb_total, w.kb0 + p.kb_per_split) - w.kb0;
  return w;
}

template <int BN, int XROWS, int KSUB>
__global__ void __launch_bounds__(kQkvThreads, 1)
    qkv_rope_kernel(const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_wq,
                    const __grid_constant__ CUtensorMap map_wk, const __grid_constant__ CUtensorMap map_wv,
                    const QkvParams p) {
  using C = QkvCfg<BN, XROWS, KSUB>;
  constexpr int kPerHead = 128 / BN;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kBarOffset);
  uint64_t* empty = full + C::kStages;
  uint64_t* acc_full = empty + C::kStages;   // [2] MMA -> epilogue
  uint64_t* acc_empty = acc_full + 2;        // [2] epilogue -> MMA
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  int32_t* flags = reinterpret_cast<int32_t*>(tmem_slot + 1);  // [0] last-CTA broadcast, [1] epilogue abort

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 4);
    }
    flags[0] = 0;
    flags[1] = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_x);
    tma_prefetch_desc(&map_wq);
    tma_prefetch_desc(&map_wk);
    tma_prefetch_desc(&map_wv);
  }
  if (warp == 1) tmem_alloc(tmem_slot, C::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // the normalised rows come from the kernel before (programmatic launch)
  pdl_wait();
  pdl_launch_dependents();
  const int units_per_head = p.n_heads * kPerHead;

  if (warp == 0) {
    // ------------------------------------------------------ TMA producer --
    if (lane == 0) {
      uint32_t g = 0;  // k-blocks issued by this CTA (ring position)
      bool ok = true;
      for (int u = blockIdx.x; u < p.n_units && ok; u += gridDim.x) {
        const QkvUnit w = qkv_unit(p, u);
        const int proj = w.n_tile / units_per_head;
        const int rem = w.n_tile % units_per_head;
        const int head = rem / kPerHead, pair = rem % kPerHead;
        const CUtensorMap* map_w = proj == 0 ? &map_wq : (proj == 1 ? &map_wk : &map_wv);
        for (int i = 0; i < w.nkb; ++i, ++g) {
          const int s = g % C::kStages;
          const uint32_t ph = (g / C::kStages) & 1;
          if (g >= static_cast<uint32_t>(C::kStages) && !mbar_wait(&empty[s], ph ^ 1, p.status, kQkvKernelId)) {
            ok = false;
            break;
          }
          uint8_t* a0 = smem + s * C::kStageBytes;
          uint8_t* b0 = a0 + C::kABytes;
          mbar_arrive_expect_tx(&full[s], C::kStageBytes);
#pragma unroll
          for (int sub = 0; sub < KSUB; ++sub) {
            uint8_t* a = a0 + sub * C::kASub;
            uint8_t* b = b0 + sub * C::kBSub;
            const int kx = ((w.kb0 + i) * KSUB + sub) * kQkvBK;
            tma_load_2d(a, &map_x, kx, w.m_tile * kQkvBM, &full[s]);
            if (BN == 128) {
              tma_load_2d(b, map_w, kx, head * 128, &full[s]);
            } else {
              tma_load_2d(b, map_w, kx, head * 128 + pair * (BN / 2), &full[s]);
              tma_load_2d(b + (BN / 2) * 128, map_w, kx, head * 128 + 64 + pair * (BN / 2), &full[s]);
            }
          }
        }
      }
    }
  } else if (warp == 1) {
    // -------------------------------------------------------- MMA issuer --
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16(kQkvBM, BN);
      uint32_t g = 0;
      int i_unit = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < p.n_units && ok; u += gridDim.x, ++i_unit) {
        const QkvUnit w = qkv_unit(p, u);
        const int acc = i_unit & 1;
        if (i_unit >= 2 && !mbar_wait(&acc_empty[acc], ((i_unit >> 1) & 1) ^ 1, p.status, kQkvKernelId)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int i = 0; i < w.nkb; ++i, ++g) {
          const int s = g % C::kStages;
          const uint32_t ph = (g / C::kStages) & 1;
          if (!mbar_wait(&full[s], ph, p.status, kQkvKernelId)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint8_t* a0 = smem + s * C::kStageBytes;
#pragma unroll
          for (int sub = 0; sub < KSUB; ++sub) {
            const uint64_t da = umma_desc_kmajor_sw128(smem_u32(a0 + sub * C::kASub));
            const uint64_t db = umma_desc_kmajor_sw128(smem_u32(a0 + C::kABytes + sub * C::kBSub));
#pragma unroll
            for (int k = 0; k < kQkvBK / 16; ++k)
              umma_bf16(d_tmem, da + 2 * k, db + 2 * k, idesc, (i > 0 || sub > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&empty[s]);
        }
        if (ok) umma_commit(&acc_full[acc]);
      }
    }
  } else {
    // ---------------------------------------------------------- epilogue --
    const int quarter = warp & 3;
    const int r_tile = quarter * 32 + lane;
    constexpr int kHalf = BN / 2;     // offset of the RoPE partner column in the tile
    constexpr int kChunks = BN / 64;  // 32-column pair chunks per tile
    const int d = p.d_model;
    int i_unit = 0;
    for (int u = blockIdx.x; u < p.n_units; u += gridDim.x, ++i_unit) {
      const QkvUnit w = qkv_unit(p, u);
      const int acc = i_unit & 1;
      const int proj = w.n_tile / units_per_head;
      const int rem = w.n_tile % units_per_head;
      const int head = rem / kPerHead, pair = rem % kPerHead;
      const int row = w.m_tile * kQkvBM + r_tile;
      const bool row_ok = row < p.n_rows;
      const uint32_t t_row = tmem_base + acc * BN + (static_cast<uint32_t>(quarter * 32) << 16);
      // Every epilogue thread reaches the named barriers (all waits are
      // bounded), so each decision below is uniform across the 4 warps.
      if (!mbar_wait(&acc_full[acc], (i_unit >> 1) & 1, p.status, kQkvKernelId)) flags[1] = 1;
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (flags[1] != 0) break;
      tc_fence_after();
      const int64_t tile_id = static_cast<int64_t>(w.n_tile) * p.m_tiles + w.m_tile;
      bool do_epilogue = true;
      if (p.splits > 1) {
        float* mine = p.partials + ((tile_id * p.splits + w.split) * kQkvBM + r_tile) * BN;
#pragma unroll
        for (int ch = 0; ch < kChunks; ++ch) {
          float a[32], b[32];
          __syncwarp();
          // warp-collective TMEM loads: every lane issues them, valid rows store
          tmem_ld_32x32b_x32(t_row + ch * 32, a);
          tmem_ld_32x32b_x32(t_row + ch * 32 + kHalf, b);
          if (row_ok) {
#pragma unroll
            for (int i = 0; i < 32; i += 4) {
              *reinterpret_cast<float4*>(mine + ch * 32 + i) = make_float4(a[i], a[i + 1], a[i + 2], a[i + 3]);
              *reinterpret_cast<float4*>(mine + ch * 32 + kHalf + i) =
                  make_float4(b[i], b[i + 1], b[i + 2], b[i + 3]);
            }
          }
        }
        __threadfence();
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (threadIdx.x == 64) {
          const int prev = atomicAdd(p.counters + tile_id, 1);
          const int last = (prev == p.splits - 1) ? 1 : 0;
          if (last) p.counters[tile_id] = 0;  // ready for the next call
          flags[0] = last;
          __threadfence();
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
        do_epilogue = flags[0] != 0;
      }
      if (do_epilogue) {
        int64_t slot = 0;
        bool slot_ok = row_ok;
        if (row_ok) {
          slot = p.pos[row];
          if (slot < 0 || slot >= p.n_slots) {
            report(p.status, FDLLM_ERR_INDEX, row, kQkvKernelId);
            slot_ok = false;
          }
        }
        __nv_bfloat16* dst = nullptr;
        if (slot_ok) {
          if (proj == 0)
            dst = p.q_out + static_cast<int64_t>(row) * d + head * 128;
          else
            dst = (proj == 1 ? p.k_out : p.v_out) + (p.kv_by_slot ? slot : static_cast<int64_t>(row)) * d +
                  head * 128;
        }
#pragma unroll
        for (int ch = 0; ch < kChunks; ++ch) {
          float a[32], b[32];
          __syncwarp();
          tmem_ld_32x32b_x32(t_row + ch * 32, a);
          tmem_ld_32x32b_x32(t_row + ch * 32 + kHalf, b);
          if (slot_ok) {
            if (p.splits > 1) {
#pragma unroll 1
              for (int s = 0; s < p.splits; ++s) {
                if (s == w.split) continue;
                const float* other = p.partials + ((tile_id * p.splits + s) * kQkvBM + r_tile) * BN;
#pragma unroll
                for (int i = 0; i < 32; i += 4) {
                  const float4 x = __ldcg(reinterpret_cast<const float4*>(other + ch * 32 + i));
                  const float4 y = __ldcg(reinterpret_cast<const float4*>(other + ch * 32 + kHalf + i));
                  a[i] += x.x; a[i + 1] += x.y; a[i + 2] += x.z; a[i + 3] += x.w;
                  b[i] += y.x; b[i + 1] += y.y; b[i + 2] += y.z; b[i + 3] += y.w;
                }
              }
            }
            const int hc = (BN == 128 ? ch * 32 : pair * 32);  // head column of a[0]; partner at hc + 64
            if (proj < 2) {
              const float* srow = p.sin + slot * 128;
              const float* crow = p.cos + slot * 128;
#pragma unroll
              for (int i = 0; i < 32; i += 4) {
                const float4 s1 = __ldg(reinterpret_cast<const float4*>(srow + hc + i));
                const float4 s2 = __ldg(reinterpret_cast<const float4*>(srow + hc + 64 + i));
                const float4 c1 = __ldg(reinterpret_cast<const float4*>(crow + hc + i));
                const float4 c2 = __ldg(reinterpret_cast<const float4*>(crow + hc + 64 + i));
                const float sa[4] = {s1.x, s1.y, s1.z, s1.w}, sb[4] = {s2.x, s2.y, s2.z, s2.w};
                const float ca[4] = {c1.x, c1.y, c1.z, c1.w}, cb[4] = {c2.x, c2.y, c2.z, c2.w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  const float x1 = a[i + j], x2 = b[i + j];
                  a[i + j] = x1 * ca[j] - x2 * sa[j];
                  b[i + j] = x2 * cb[j] + x1 * sb[j];
                }
              }
            }
#pragma unroll
            for (int i = 0; i < 32; i += 8) {
              uint4 va, vb;
              va.x = pack_bf16x2(a[i], a[i + 1]);
              va.y = pack_bf16x2(a[i + 2], a[i + 3]);
              va.z = pack_bf16x2(a[i + 4], a[i + 5]);
              va.w = pack_bf16x2(a[i + 6], a[i + 7]);
              vb.x = pack_bf16x2(b[i], b[i + 1]);
              vb.y = pack_bf16x2(b[i + 2], b[i + 3]);
              vb.z = pack_bf16x2(b[i + 4], b[i + 5]);
              vb.w = pack_bf16x2(b[i + 6], b[i + 7]);
              *reinterpret_cast<uint4*>(dst + hc + i) = va;
              *reinterpret_cast<uint4*>(dst + hc + 64 + i) = vb;
            }
          }
        }
      }
      // this accumulator may now be overwritten by the unit after next
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[acc]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// CTA-pair variant (more than 128 rows).  A cluster of two CTAs computes
// 256-row x 256-column tiles (two heads; the last tile of an odd head count
// is one head) with 2-SM UMMAs (cta_group::2, M = 256): CTA r loads rows
// 128r..128r+127 of the tile's X rows and head h0 + r of its W rows (rows
// 64r..64r+63 of a one-head tile), and holds its 128 output rows in its own
// TMEM.  Each SM then moves 512 operand bytes per 64K flops of a k-step,
// which keeps it under the ~108 GB/s an SM pulls from L2 through TMA.
//
// Work is split stream-K: the (tile, k-block) iterations are cut into one
// contiguous range per pair.  A range that starts inside a tile contributes
// that tile's last k-blocks first and stores the partial accumulator (fp32,
// one slot per pair) with a release flag; the pair whose range holds the
// tile's k-block 0 does that tile last, adds the partials of the pairs after
// it and runs the epilogue.  Owners only wait on pairs of higher index that
// did their part first, on a grid that is resident all at once.
//
// Rank 0 issues the MMAs; the leader's `full` barrier expects the bytes of
// both CTAs' loads, which complete their transactions on it (plain loads, no
// multicast); stage and accumulator completions are committed to both CTAs.
// Warpgroup 0 holds the TMA producer and MMA warps and gives registers up
// (setmaxnreg 48) to warpgroups 1-2, the eight epilogue warps (224 each, two
// per TMEM lane quarter), which move each 32-column slice
// and its RoPE partner slice 64 columns on from TMEM through a swizzled fp32
// staging buffer, so that the RoPE tables are read and the outputs written
// row-contiguously, sixteen rows per warp in one batch of loads.  The last
// segment's epilogue is not hidden behind MMAs: it first copies the RoPE
// rows of its 128 rows into the (then idle) operand ring with cp.async and
// reads them from there.
// ---------------------------------------------------------------------------
constexpr int kQ2ABytes = kQkvBM * kQkvBK * 2;                // 128 X rows x 64 K
constexpr int kQ2BHalfBytes = 64 * kQkvBK * 2;                // 64 W rows x 64 K
constexpr int kQ2StageBytes = kQ2ABytes + 2 * kQ2BHalfBytes;  // 32 KB
constexpr int kQ2Stages = 6;
constexpr int kQ2StagingOffset = kQ2Stages * kQ2StageBytes;
constexpr int kQ2StagingBytes = kQkvBM * 64 * 4;  // 128 rows x (32 + 32) fp32
constexpr int kQ2BarOffset = kQ2StagingOffset + kQ2StagingBytes;
constexpr int kQ2Smem = 1024 + kQ2BarOffset + 256;
constexpr int kQ2AccCols = 256;
constexpr int kQ2TmemCols = 2 * kQ2AccCols;          // double-buffered accumulator
constexpr int kQ2PartialFloats = kQkvBM * kQ2AccCols;  // one CTA's partial accumulator
constexpr int kQ2Threads = 384;  // warpgroup 0: producer, MMA, 2 idle; warpgroups 1-2: epilogue
// Register split: 128 x 48 + 256 x 224 <= 384 x 168 at launch.
constexpr int kQ2RegsLow = 48, kQ2RegsHigh = 224;
static_assert(128 * kQ2RegsLow + 256 * kQ2RegsHigh <= kQ2Threads * 168, "setmaxnreg split");
static_assert(kQ2Smem <= 232448, "CTA-pair QKV shared memory");

struct Q2Seg {
  int tile, k0, k1;  // k-blocks [k0, k1) of `tile`
};

__device__ __forceinline__ int q2_lo(int pair, int n_pairs, int iters) {
  return static_cast<int>(static_cast<long long>(pair) * iters / n_pairs);
}

// Segment k of the iteration range [lo, hi) (k < q2_nsegs): the k-blocks of
// one tile, in range order.
__device__ __forceinline__ int q2_nsegs(int lo, int hi, int kbt) { return lo < hi ? (hi - 1) / kbt - lo / kbt + 1 : 0; }

__device__ __forceinline__ Q2Seg q2_seg_at(int lo, int hi, int kbt, int k) {
  Q2Seg s;
  s.tile = lo / kbt + k;
  s.k0 = k == 0 ? lo % kbt : 0;
  const int end = hi - s.tile * kbt;
  s.k1 = end < kbt ? end : kbt;
  return s;
}

// Next segment of the iteration range [i, hi): the k-blocks of one tile.
__device__ __forceinline__ bool q2_next(int& i, int hi, int kbt, Q2Seg& s) {
  if (i >= hi) return false;
  s.tile = i / kbt;
  s.k0 = i % kbt;
  s.k1 = s.k0 + (hi - i) < kbt ? s.k0 + (hi - i) : kbt;
  i += s.k1 - s.k0;
  return true;
}

// RoPE + bf16 store of 16 staged rows of one 32-column slice (and its
// partners 64 columns on): half-warp hw of the warp takes rows 2k + hw of its
// 16, lane j the columns c, c + 1, with the RoPE rows read from the tables by
// slot and the outputs written to `out` (head column 0) by row or slot.  Rows
// whose slot is negative are not written.
__device__ __forceinline__ void q2_rope_rows(const float* staging, const QkvParams& p, int quarter, int half, int hw,
                                             int j, int c, bool rope, int64_t my_slot, __nv_bfloat16* out, int d,
                                             bool by_slot, int row_base) {
  float2 y1[8], y2[8];
  int64_t sl[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int rr = half * 16 + 2 * k + hw;  // row within the warp's quarter
    const int rt = quarter * 32 + rr;
    sl[k] = __shfl_sync(0xffffffffu, my_slot, rr);
    const float* st = staging + rt * 64;
    const int pu = (j >> 1) ^ (rt & 7);
    const float2 x1 = *reinterpret_cast<const float2*>(st + pu * 4 + (j & 1) * 2);
    const float2 x2 = *reinterpret_cast<const float2*>(st + 32 + pu * 4 + (j & 1) * 2);
    y1[k] = x1;
    y2[k] = x2;
    if (rope) {
      const int64_t sr = sl[k] < 0 ? 0 : sl[k];  // invalid rows read slot 0 and are not stored
      const float2 s1 = __ldg(reinterpret_cast<const float2*>(p.sin + sr * 128 + c));
      const float2 s2 = __ldg(reinterpret_cast<const float2*>(p.sin + sr * 128 + c + 64));
      const float2 c1 = __ldg(reinterpret_cast<const float2*>(p.cos + sr * 128 + c));
      const float2 c2 = __ldg(reinterpret_cast<const float2*>(p.cos + sr * 128 + c + 64));
      y1[k].x = x1.x * c1.x - x2.x * s1.x;
      y1[k].y = x1.y * c1.y - x2.y * s1.y;
      y2[k].x = x2.x * c2.x + x1.x * s2.x;
      y2[k].y = x2.y * c2.y + x1.y * s2.y;
    }
  }
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int rt = quarter * 32 + half * 16 + 2 * k + hw;
    if (sl[k] >= 0) {
      const int64_t orow = by_slot ? sl[k] : static_cast<int64_t>(row_base + rt);
      __nv_bfloat16* dst = out + orow * d;
      *reinterpret_cast<uint32_t*>(dst + c) = pack_bf16x2(y1[k].x, y1[k].y);
      *reinterpret_cast<uint32_t*>(dst + c + 64) = pack_bf16x2(y2[k].x, y2[k].y);
    }
  }
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kQ2Threads, 1)
    qkv2_rope_kernel(const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_wq,
                     const __grid_constant__ CUtensorMap map_wk, const __grid_constant__ CUtensorMap map_wv,
                     const QkvParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* staging = reinterpret_cast<float*>(smem + kQ2StagingOffset);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kQ2BarOffset);
  uint64_t* empty = full + kQ2Stages;
  uint64_t* acc_full = empty + kQ2Stages;  // [2] MMA -> epilogue (both CTAs)
  uint64_t* acc_empty = acc_full + 2;      // [2] epilogues of both CTAs -> MMA (leader's)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  int32_t* abort_flag = reinterpret_cast<int32_t*>(tmem_slot + 1);
  uint64_t* tab_bar = acc_empty + 3;  // last segment: RoPE rows landed (256 arrivals)

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int pair_id = blockIdx.x >> 1;
  const int n_pairs = gridDim.x >> 1;
  const int m_pairs = (p.n_rows + 2 * kQkvBM - 1) / (2 * kQkvBM);
  const int n_blocks = 3 * p.n_heads;
  const int kbt = p.d_model / kQkvBK;
  const int iters = m_pairs * ((n_blocks + 1) / 2) * kbt;
  const int lo = q2_lo(pair_id, n_pairs, iters);
  const int hi = q2_lo(pair_id + 1, n_pairs, iters);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kQ2Stages; ++s) {
      mbar_init(&full[s], 1);   // the leader's expect_tx arrival (used on the leader)
      mbar_init(&empty[s], 1);  // the leader's commit
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 16);  // 8 epilogue warps x 2 CTAs (used on the leader)
    }
    mbar_init(tab_bar, 256);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_x);
    tma_prefetch_desc(&map_wq);
    tma_prefetch_desc(&map_wk);
    tma_prefetch_desc(&map_wv);
  }
  if (warp == 1) tmem_alloc_pair(tmem_slot, kQ2TmemCols);
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers exist before any remote arrival
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // the normalised rows come from the kernel before (programmatic launch)
  pdl_wait();
  pdl_launch_dependents();
  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kQ2RegsLow));
  if (warp == 0) {
    // ------------------------------------------------------ TMA producer --
    if (lane == 0) {
      uint32_t g = 0;
      bool ok = true;
      int i = lo;
      Q2Seg sg;
      while (ok && q2_next(i, hi, kbt, sg)) {
        const int m_pair = sg.tile % m_pairs, b = (sg.tile / m_pairs) * 2;
        const int nblk = n_blocks - b < 2 ? n_blocks - b : 2;
        // W rows this CTA loads: head b + rank (two heads) or half `rank` of head b
        const int head_g = nblk == 2 ? b + static_cast<int>(rank) : b;
        const int proj = head_g / p.n_heads;
        const int w_row = (head_g % p.n_heads) * 128 + (nblk == 2 ? 0 : static_cast<int>(rank) * 64);
        const CUtensorMap* map_w = proj == 0 ? &map_wq : (proj == 1 ? &map_wk : &map_wv);
        const uint32_t tx = 2u * static_cast<uint32_t>(kQ2ABytes + nblk * kQ2BHalfBytes);
        const int x_row = m_pair * 2 * kQkvBM + static_cast<int>(rank) * kQkvBM;
        for (int kb = sg.k0; kb < sg.k1; ++kb, ++g) {
          const int s = g % kQ2Stages;
          const uint32_t ph = (g / kQ2Stages) & 1;
          if (g >= static_cast<uint32_t>(kQ2Stages) && !mbar_wait(&empty[s], ph ^ 1, p.status, kQkvKernelId)) {
            ok = false;
            break;
          }
          uint8_t* a = smem + s * kQ2StageBytes;
          const uint32_t bar = mapa_shared(&full[s], 0);
          // the leader expects both CTAs' bytes; the peer's loads only
          // complete transactions on it (a cluster-scope arrive per stage
          // costs about one load latency, serialising the ring)
          if (rank == 0) mbar_arrive_expect_tx(&full[s], tx);
          tma_load_2d_pair(a, &map_x, kb * kQkvBK, x_row, bar);
          tma_load_2d_pair(a + kQ2ABytes, map_w, kb * kQkvBK, w_row, bar);
          if (nblk == 2) tma_load_2d_pair(a + kQ2ABytes + kQ2BHalfBytes, map_w, kb * kQkvBK, w_row + 64, bar);
        }
      }
    }
  } else if (warp == 1) {
    // -------------------------------------------- MMA issuer (leader only) --
    if (rank == 0 && lane == 0) {
      constexpr uint32_t idesc1 = umma_idesc_bf16(2 * kQkvBM, 128);
      constexpr uint32_t idesc2 = umma_idesc_bf16(2 * kQkvBM, 256);
      uint32_t g = 0;
      int i_unit = 0;
      bool ok = true;
      int i = lo;
      Q2Seg sg;
      while (ok && q2_next(i, hi, kbt, sg)) {
        const int b = (sg.tile / m_pairs) * 2;
        const uint32_t idesc = n_blocks - b < 2 ? idesc1 : idesc2;
        const int acc = i_unit & 1;
        if (i_unit >= 2 && !mbar_wait(&acc_empty[acc], ((i_unit >> 1) & 1) ^ 1, p.status, kQkvKernelId)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kQ2AccCols;
        for (int kb = sg.k0; kb < sg.k1; ++kb, ++g) {
          const int s = g % kQ2Stages;
          const uint32_t ph = (g / kQ2Stages) & 1;
          if (!mbar_wait(&full[s], ph, p.status, kQkvKernelId)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint8_t* a = smem + s * kQ2StageBytes;
          const uint64_t da = umma_desc_kmajor_sw128(smem_u32(a));
          const uint64_t db = umma_desc_kmajor_sw128(smem_u32(a + kQ2ABytes));
#pragma unroll
          for (int k = 0; k < kQkvBK / 16; ++k)
            umma_bf16_pair(d_tmem, da + 2 * k, db + 2 * k, idesc, (kb > sg.k0 || k > 0) ? 1u : 0u);
          umma_commit_pair(mapa_shared(&empty[s], 0));
          umma_commit_pair(mapa_shared(&empty[s], 1));
        }
        if (!ok) break;
        umma_commit_pair(mapa_shared(&acc_full[acc], 0));
        umma_commit_pair(mapa_shared(&acc_full[acc], 1));
        ++i_unit;
      }
    }
  }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kQ2RegsHigh));
    // ---------------------------------------------------------- epilogue --
    const int quarter = warp & 3;
    const int half = (warp - 4) >> 2;        // 0: a-columns / first 16 rows, 1: partner columns / last 16
    const int r_tile = quarter * 32 + lane;  // this thread's TMEM lane / tile row
    const int ep_tid = threadIdx.x - 128;
    const int d = p.d_model;
    // Epilogues run in range order, except that an owner part ending the
    // range is finished before the whole tile in front of it: both then run
    // after the last MMA, with the ring idle (thread-per-row path).
    const int n_segs = q2_nsegs(lo, hi, kbt);
    bool swap_last = false;
    if (n_segs >= 2) {
      const Q2Seg s_last = q2_seg_at(lo, hi, kbt, n_segs - 1), s_prev = q2_seg_at(lo, hi, kbt, n_segs - 2);
      swap_last = s_last.k1 < kbt && s_prev.k0 == 0 && s_prev.k1 == kbt;
    }
    uint32_t tab_phase = 0;
    for (int e = 0; e < n_segs; ++e) {
      const int m_idx = (swap_last && e >= n_segs - 2) ? 2 * n_segs - 3 - e : e;  // MMA order of the segment
      const Q2Seg sg = q2_seg_at(lo, hi, kbt, m_idx);
      const bool last = e == n_segs - 1 || (swap_last && e == n_segs - 2);  // after the last MMA
      const int m_pair = sg.tile % m_pairs, b = (sg.tile / m_pairs) * 2;
      const int nblk = n_blocks - b < 2 ? n_blocks - b : 2;
      const int acc = m_idx & 1;
      const uint32_t t_base = tmem_base + acc * kQ2AccCols + (static_cast<uint32_t>(quarter * 32) << 16);
      // row slot, and its RoPE rows pulled into L2 while the MMAs run (the
      // epilogue's table reads are otherwise serialised DRAM round trips)
      const int row_base = m_pair * 2 * kQkvBM + static_cast<int>(rank) * kQkvBM;
      int64_t my_slot = -1;  // slot of row r_tile; -1: row not written
      if (sg.k0 == 0 && row_base + r_tile < p.n_rows) {
        const int64_t s = p.pos[row_base + r_tile];
        if (s < 0 || s >= p.n_slots) {
          report(p.status, FDLLM_ERR_INDEX, row_base + r_tile, kQkvKernelId);
        } else {
          my_slot = s;
          if (b / p.n_heads < 2) {
            const float* tab = half == 0 ? p.sin : p.cos;
#pragma unroll
            for (int l = 0; l < 128; l += 32) asm volatile("prefetch.global.L2 [%0];" ::"l"(tab + s * 128 + l));
          }
        }
      }
      if (!mbar_wait(&acc_full[acc], (m_idx >> 1) & 1, p.status, kQkvKernelId)) *abort_flag = 1;
      asm volatile("bar.sync 1, 256;" ::: "memory");
      if (*abort_flag != 0) break;
      tc_fence_after();
      if (sg.k0 > 0) {
        // contributor: store the partial sums ([col / 4][row][4] fp32, so a
        // warp's accesses are 512 contiguous bytes) and publish them
        float4* part = reinterpret_cast<float4*>(p.partials) + static_cast<size_t>(pair_id * 2 + rank) *
                                                                  (kQ2PartialFloats / 4);
        for (int c = half * 32; c < nblk * 128; c += 64) {
          float v[32];
          __syncwarp();
          tmem_ld_32x32b_x32(t_base + c, v);
#pragma unroll
          for (int j = 0; j < 32; j += 4)
            __stcg(part + ((c + j) >> 2) * kQkvBM + r_tile, make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]));
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(mapa_shared(&acc_empty[acc], 0));
        __threadfence();
        asm volatile("bar.sync 1, 256;" ::: "memory");
        if (ep_tid == 0) st_release_gpu(p.counters + pair_id * 2 + rank, 1);
        continue;
      }
      // a whole tile, or the owner's part (k-block 0 on): add the partials of
      // the pairs whose ranges start inside this tile
      int q_end = pair_id + 1;
      if (sg.k1 < kbt) {
        const int t_end = (sg.tile + 1) * kbt;
        while (q_end < n_pairs && q2_lo(q_end, n_pairs, iters) < t_end) ++q_end;
        for (int q = pair_id + 1; q < q_end; ++q) flag_wait_set(p.counters + q * 2 + rank, p.status, kQkvKernelId);
      }
      const bool rope_tile = b / p.n_heads < 2;  // the tile has a Q or K head
      if (last) {
        // The last segment's epilogue is not hidden behind MMAs, and the ring
        // is idle then (every MMA that read it has completed).  It runs
        // thread-per-row straight from TMEM: the rows' RoPE tables are
        // bulk-copied into the ring with a 1040-byte row stride (a warp's
        // 16-byte reads of 32 rows then spread over all bank groups), the
        // contributor's partial sums (if any) come by coalesced loads, and
        // the bf16 rows are staged (272-byte stride) and leave by one 256-byte
        // bulk store per row and head.  Half h takes head columns 32h..32h+31
        // and their partners 64 + 32h.. of every head.
        constexpr int kTabStride = 1040, kOutStride = 272;
        uint8_t* tabs = smem;                        // row r: sin[128] | cos[128] fp32
        uint8_t* outs = smem + kQkvBM * kTabStride;  // head hh, row r: 128 bf16
        if (rope_tile) {
          mbar_arrive_expect_tx(tab_bar, my_slot >= 0 ? 512u : 0u);
          if (my_slot >= 0)
            bulk_load(tabs + r_tile * kTabStride + half * 512, (half == 0 ? p.sin : p.cos) + my_slot * 128, 512,
                      tab_bar);
        }
        bool tabs_ready = false;
        for (int hh = 0; hh < nblk; ++hh) {
          const int proj = (b + hh) / p.n_heads;
#pragma unroll 1
          for (int g = 0; g < 2; ++g) {
            const int cg = half * 32 + g * 16;  // head column of a[0]; RoPE partners at cg + 64
            const int ca = hh * 128 + cg;
            float a[16], bv[16];
            __syncwarp();
            tmem_ld_32x32b_x16(t_base + ca, a);
            tmem_ld_32x32b_x16(t_base + ca + 64, bv);
            for (int q = pair_id + 1; q < q_end; ++q) {
              const float4* part = reinterpret_cast<const float4*>(p.partials) +
                                   static_cast<size_t>(q * 2 + rank) * (kQ2PartialFloats / 4);
#pragma unroll
              for (int j = 0; j < 16; j += 4) {
                const float4 x = __ldcg(part + ((ca + j) >> 2) * kQkvBM + r_tile);
                const float4 y = __ldcg(part + ((ca + 64 + j) >> 2) * kQkvBM + r_tile);
                a[j] += x.x;
                a[j + 1] += x.y;
                a[j + 2] += x.z;
                a[j + 3] += x.w;
                bv[j] += y.x;
                bv[j + 1] += y.y;
                bv[j + 2] += y.z;
                bv[j + 3] += y.w;
              }
            }
            if (hh == nblk - 1 && g == 1) {
              // every column of this accumulator has been read
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive_cluster(mapa_shared(&acc_empty[acc], 0));
            }
            if (proj < 2 && my_slot >= 0) {
              if (!tabs_ready) {
                mbar_wait(tab_bar, tab_phase & 1, p.status, kQkvKernelId);
                tabs_ready = true;
              }
              const uint8_t* trow = tabs + r_tile * kTabStride + cg * 4;
#pragma unroll
              for (int i = 0; i < 16; i += 4) {
                const float4 s1 = *reinterpret_cast<const float4*>(trow + i * 4);
                const float4 s2 = *reinterpret_cast<const float4*>(trow + 256 + i * 4);
                const float4 c1 = *reinterpret_cast<const float4*>(trow + 512 + i * 4);
                const float4 c2 = *reinterpret_cast<const float4*>(trow + 768 + i * 4);
                const float sa[4] = {s1.x, s1.y, s1.z, s1.w}, sb[4] = {s2.x, s2.y, s2.z, s2.w};
                const float ca4[4] = {c1.x, c1.y, c1.z, c1.w}, cb4[4] = {c2.x, c2.y, c2.z, c2.w};
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                  const float x1 = a[i + k], x2 = bv[i + k];
                  a[i + k] = x1 * ca4[k] - x2 * sa[k];
                  bv[i + k] = x2 * cb4[k] + x1 * sb[k];
                }
              }
            }
            uint8_t* orow = outs + (hh * kQkvBM + r_tile) * kOutStride + cg * 2;
#pragma unroll
            for (int i = 0; i < 16; i += 8) {
              uint4 va, vb;
              va.x = pack_bf16x2(a[i], a[i + 1]);
              va.y = pack_bf16x2(a[i + 2], a[i + 3]);
              va.z = pack_bf16x2(a[i + 4], a[i + 5]);
              va.w = pack_bf16x2(a[i + 6], a[i + 7]);
              vb.x = pack_bf16x2(bv[i], bv[i + 1]);
              vb.y = pack_bf16x2(bv[i + 2], bv[i + 3]);
              vb.z = pack_bf16x2(bv[i + 4], bv[i + 5]);
              vb.w = pack_bf16x2(bv[i + 6], bv[i + 7]);
              *reinterpret_cast<uint4*>(orow + i * 2) = va;
              *reinterpret_cast<uint4*>(orow + 128 + i * 2) = vb;
            }
          }
        }
        if (rope_tile && !tabs_ready) mbar_wait(tab_bar, tab_phase & 1, p.status, kQkvKernelId);  // no copy in flight
        if (rope_tile) ++tab_phase;
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        asm volatile("bar.sync 1, 256;" ::: "memory");
        if (half == 0 && my_slot >= 0) {
          for (int hh = 0; hh < nblk; ++hh) {
            const int head_g = b + hh;
            const int proj = head_g / p.n_heads, head = head_g % p.n_heads;
            __nv_bfloat16* out = proj == 0 ? p.q_out : (proj == 1 ? p.k_out : p.v_out);
            const int64_t orow_g = (proj > 0 && p.kv_by_slot) ? my_slot : static_cast<int64_t>(row_base + r_tile);
            bulk_store(out + orow_g * d + head * 128, outs + (hh * kQkvBM + r_tile) * kOutStride, 256);
          }
          bulk_commit();
          bulk_wait_all();
        }
        asm volatile("bar.sync 1, 256;" ::: "memory");  // the staged rows were read: tables / rows reusable
      } else {
        for (int hh = 0; hh < nblk; ++hh) {
          const int head_g = b + hh;
          const int proj = head_g / p.n_heads, head = head_g % p.n_heads;
          __nv_bfloat16* out = proj == 0 ? p.q_out : (proj == 1 ? p.k_out : p.v_out);
          const bool by_slot = proj > 0 && p.kv_by_slot;
          for (int sub = 0; sub < 2; ++sub) {
            // half 0 takes columns ca.., half 1 their RoPE partners ca + 64..
            const int ca = hh * 128 + sub * 32 + half * 64;
            float a[32];
            __syncwarp();
            tmem_ld_32x32b_x32(t_base + ca, a);
            for (int q = pair_id + 1; q < q_end; ++q) {
              const float4* part = reinterpret_cast<const float4*>(p.partials) +
                                   static_cast<size_t>(q * 2 + rank) * (kQ2PartialFloats / 4);
#pragma unroll
              for (int j = 0; j < 32; j += 4) {
                const float4 x = __ldcg(part + ((ca + j) >> 2) * kQkvBM + r_tile);
                a[j] += x.x;
                a[j + 1] += x.y;
                a[j + 2] += x.z;
                a[j + 3] += x.w;
              }
            }
            if (hh == nblk - 1 && sub == 1) {
              // every column of this accumulator has been read
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive_cluster(mapa_shared(&acc_empty[acc], 0));
            }
            // stage row r_tile: a-columns -> 16-byte units 0..7, partners ->
            // 8..15, unit ^ (row & 7)
            float* srow = staging + r_tile * 64 + half * 32;
#pragma unroll
            for (int u = 0; u < 8; ++u) {
              const int pu = u ^ (r_tile & 7);
              *reinterpret_cast<float4*>(srow + pu * 4) =
                  make_float4(a[4 * u], a[4 * u + 1], a[4 * u + 2], a[4 * u + 3]);
            }
            asm volatile("bar.sync 1, 256;" ::: "memory");
            // 16 rows of this warp's quarter, two per step: half-warp h takes
            // row 2k + h, lane j = lane & 15 takes head columns c, c + 1
            // (c = sub * 32 + 2j) and their partners c + 64, c + 65
            q2_rope_rows(staging, p, quarter, half, lane >> 4, lane & 15, sub * 32 + 2 * (lane & 15), proj < 2,
                         my_slot, out + head * 128, d, by_slot, row_base);
            asm volatile("bar.sync 1, 256;" ::: "memory");  // staging free again
          }
        }
      }
      // the partials were read by every epilogue thread (the barrier above):
      // clear the contributors' flags for the next launch
      if (ep_tid == 0)
        for (int q = pair_id + 1; q < q_end; ++q) p.counters[q * 2 + rank] = 0;
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // the leader's MMAs read both CTAs' shared memory until here
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kQ2TmemCols);
  }
}

namespace {

struct QkvPlan {
  int bn;
  int xrows;
  int ksub;
  int splits;
  int kb_per_split;
  int m_tiles;
  int n_tiles;
  int n_units;
  int grid;
  bool pair;  // CTA-pair stream-K kernel (more than 128 rows)
};

// Plan overrides for tuning and tests (fdllm_qkv_set_plan); 0 / -1 mean
// automatic.  The first values come from FDLLM_QKV_BN / FDLLM_QKV_SPLITS /
// FDLLM_QKV_KSUB / FDLLM_QKV_PAIR, read once per process.
struct QkvOverride {
  int impl, bn, splits, ksub, pair;
};

QkvOverride& qkv_override() {
  static QkvOverride o{env_int("FDLLM_QKV_IMPL", -1), env_int("FDLLM_QKV_BN", 0), env_int("FDLLM_QKV_SPLITS", 1),
                       env_int("FDLLM_QKV_KSUB", 0), env_int("FDLLM_QKV_PAIR", -1)};
  return o;
}

// Kernel choice: the stream-K GEMM at every row count (back to back with the
// weights streaming from HBM: 64 rows 24.9 vs 25.2 us, 128 rows 28.0 vs
// 30.6 us, 512 rows 55 vs 58 us against the whole-tile kernels), unless
// overridden.
bool qkv_use_sk(int32_t n_rows) {
  (void)n_rows;
  return qkv_override().impl != 1;
}

// Units are spread round-robin over one CTA per SM.  Tiles are 128 columns
// (one head) wide and K is not split by default: at 64 and 128 rows (96
// tiles) whole-K tiles on 96 SMs measured faster than 64-wide tiles on all
// SMs (64 rows: 35.5 vs 39.6 us) and than 2-6 K splits, whose fp32 partials
// cost more than the balance gains (64 rows: 41.7-92 us).
QkvPlan plan_qkv(int32_t n_rows, int32_t d_model, int32_t n_heads) {
  QkvPlan pl{};
  const QkvOverride& ov = qkv_override();
  int ksub = ov.ksub;
  if (ksub != 1 && ksub != 2) ksub = 2;
  if (d_model % (kQkvBK * ksub) != 0) ksub = 1;
  pl.ksub = ksub;
  const int kb_total = d_model / (kQkvBK * ksub);
  const int sms = sm_count();
  pl.m_tiles = (n_rows + kQkvBM - 1) / kQkvBM;
  pl.xrows = n_rows <= 64 ? 64 : 128;
  int bn = ov.bn;
  if (bn != 64 && bn != 128) bn = 128;
  pl.bn = bn;
  pl.n_tiles = 3 * n_heads * (128 / bn);
  const int tiles = pl.m_tiles * pl.n_tiles;
  int splits = ov.splits;
  if (splits < 1) splits = 1;
  if (splits > kb_total) splits = kb_total;
  pl.kb_per_split = (kb_total + splits - 1) / splits;
  pl.splits = (kb_total + pl.kb_per_split - 1) / pl.kb_per_split;  // no empty splits
  pl.n_units = tiles * pl.splits;
  pl.grid = pl.n_units < sms ? pl.n_units : sms;
  // CTA pairs for 129-256 rows, where they measured faster (256 rows: 45.9
  // vs 51.1 us; 384 and 512 rows: 69 vs 55-66 us).  FDLLM_QKV_PAIR=1 / 0
  // forces them on above 128 rows / off.
  const int pair_env = ov.pair;
  pl.pair = n_rows > 128 && d_model % kQkvBK == 0 && (pair_env < 0 ? n_rows <= 256 : pair_env != 0);
  if (pl.pair) {
    pl.splits = 1;
    pl.kb_per_split = d_model / (kQkvBK * pl.ksub);
    pl.bn = 128;
    pl.xrows = 128;
    pl.grid = 2 * (sms / 2);  // capped at the resident pairs at launch
  }
  return pl;
}

// Workspace layout: a fixed counter region (so counters never move between
// calls with different tile counts, and no call's partial sums land on another
// call's counters), then the split-K partials.
constexpr size_t kQkvCounterBytes = 4096;  // 1024 tiles (K splits are requested through FDLLM_QKV_SPLITS)

size_t qkv_ws_bytes(const QkvPlan& pl) {
  // CTA pairs: flags, then one partial accumulator slot per CTA
  if (pl.pair) return kQkvCounterBytes + static_cast<size_t>(pl.grid) * kQ2PartialFloats * sizeof(float);
  if (pl.splits <= 1) return 256;
  const size_t tiles = static_cast<size_t>(pl.m_tiles) * pl.n_tiles;
  return kQkvCounterBytes + tiles * pl.splits * kQkvBM * pl.bn * sizeof(float);
}

template <int BN, int XROWS, int KSUB>
int launch_qkv_cfg(const CUtensorMap& mx, const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
                   const QkvParams& p, const QkvPlan& pl, cudaStream_t stream) {
  using C = QkvCfg<BN, XROWS, KSUB>;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_set[dev]) {
    if (cudaFuncSetAttribute(qkv_rope_kernel<BN, XROWS, KSUB>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem) !=
        cudaSuccess)
      return FDLLM_ERR_CUDA;
    attr_set[dev] = true;
  }
  if (launch_ex(qkv_rope_kernel<BN, XROWS, KSUB>, dim3(pl.grid), dim3(kQkvThreads), C::kSmem, stream, 1,
                pdl_enabled(), mx, mq, mk, mv, p) != cudaSuccess)
    return FDLLM_ERR_CUDA;
  return cudaPeekAtLastError() == cudaSuccess ? FDLLM_OK : FDLLM_ERR_CUDA;
}

int launch_qkv(const void* xn, const void* wq, const void* wk, const void* wv, const int64_t* pos,
               const float* rope_sin, const float* rope_cos, void* q_out, void* k_out, void* v_out,
               int32_t n_rows, int32_t d_model, int32_t n_heads, int64_t n_slots, void* workspace,
               size_t workspace_bytes, int kv_by_slot, cudaStream_t stream) {
  if (n_rows < 0 || n_heads <= 0 || d_model != n_heads * 128 || n_slots <= 0) return FDLLM_ERR_ARG;
  if (n_rows == 0) return FDLLM_OK;
  const void* ptrs[] = {xn, wq, wk, wv, pos, rope_sin, rope_cos, q_out, k_out, v_out};
  for (const void* q : ptrs)
    if (q == nullptr || !aligned16(q)) return FDLLM_ERR_ARG;
  const QkvPlan pl = plan_qkv(n_rows, d_model, n_heads);
  if ((pl.splits > 1 || pl.pair) && (workspace == nullptr || workspace_bytes < qkv_ws_bytes(pl)))
    return FDLLM_ERR_WORKSPACE;
  CUtensorMap mx, mq, mk, mv;
  int rc;
  if ((rc = make_tmap_bf16_sw128(&mx, xn, n_rows, d_model, d_model, pl.xrows)) != FDLLM_OK) return rc;
  const uint32_t wbox = pl.pair ? 64 : (pl.bn == 128 ? 128 : pl.bn / 2);
  if ((rc = make_tmap_bf16_sw128(&mq, wq, d_model, d_model, d_model, wbox)) != FDLLM_OK) return rc;
  if ((rc = make_tmap_bf16_sw128(&mk, wk, d_model, d_model, d_model, wbox)) != FDLLM_OK) return rc;
  if ((rc = make_tmap_bf16_sw128(&mv, wv, d_model, d_model, d_model, wbox)) != FDLLM_OK) return rc;
  QkvParams p{};
  p.pos = pos;
  p.sin = rope_sin;
  p.cos = rope_cos;
  p.q_out = static_cast<__nv_bfloat16*>(q_out);
  p.k_out = static_cast<__nv_bfloat16*>(k_out);
  p.v_out = static_cast<__nv_bfloat16*>(v_out);
  p.status = status_ptr();
  p.n_slots = n_slots;
  p.n_rows = n_rows;
  p.d_model = d_model;
  p.n_heads = n_heads;
  p.kv_by_slot = kv_by_slot;
  p.splits = pl.splits;
  p.kb_per_split = pl.kb_per_split;
  p.m_tiles = pl.m_tiles;
  p.n_units = pl.n_units;
  p.ksub = pl.ksub;
  if (pl.pair) {
    if (static_cast<size_t>(pl.grid) * sizeof(int32_t) > kQkvCounterBytes) return FDLLM_ERR_ARG;
    p.counters = static_cast<int32_t*>(workspace);
    p.partials = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + kQkvCounterBytes);
  } else if (pl.splits > 1) {
    if (static_cast<size_t>(pl.m_tiles) * pl.n_tiles * sizeof(int32_t) > kQkvCounterBytes) return FDLLM_ERR_ARG;
    p.counters = static_cast<int32_t*>(workspace);
    p.partials = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + kQkvCounterBytes);
  }
  if (pl.pair) {
    // One pair per two SMs, capped at the number of pairs that are resident
    // at once (a GPC with an odd SM count leaves one SM out).
    static int max_pairs[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 64) return FDLLM_ERR_ARG;
    if (max_pairs[dev] == 0) {
      if (cudaFuncSetAttribute(qkv2_rope_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kQ2Smem) != cudaSuccess)
        return FDLLM_ERR_CUDA;
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(static_cast<unsigned>(pl.grid), 1, 1);
      cfg.blockDim = dim3(kQ2Threads, 1, 1);
      cfg.dynamicSmemBytes = kQ2Smem;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, qkv2_rope_kernel, &cfg) != cudaSuccess || n <= 0) return FDLLM_ERR_CUDA;
      max_pairs[dev] = n;
    }
    // every pair gets a non-empty iteration range; all pairs are resident
    // at once (owners wait on the partials of later pairs)
    const long long iters = static_cast<long long>((n_rows + 2 * kQkvBM - 1) / (2 * kQkvBM)) *
                            ((3 * n_heads + 1) / 2) * (d_model / kQkvBK);
    int pairs = pl.grid / 2 < max_pairs[dev] ? pl.grid / 2 : max_pairs[dev];
    if (iters < pairs) pairs = static_cast<int>(iters);
    if (iters > (1ll << 30)) return FDLLM_ERR_ARG;
    if (launch_ex(qkv2_rope_kernel, dim3(2 * pairs), dim3(kQ2Threads), kQ2Smem, stream, 1, pdl_enabled(), mx, mq,
                  mk, mv, p) != cudaSuccess)
      return FDLLM_ERR_CUDA;
    return cudaPeekAtLastError() == cudaSuccess ? FDLLM_OK : FDLLM_ERR_CUDA;
  }
  if (pl.ksub == 2) {
    if (pl.bn == 128)
      return pl.xrows == 64 ? launch_qkv_cfg<128, 64, 2>(mx, mq, mk, mv, p, pl, stream)
                            : launch_qkv_cfg<128, 128, 2>(mx, mq, mk, mv, p, pl, stream);
    return pl.xrows == 64 ? launch_qkv_cfg<64, 64, 2>(mx, mq, mk, mv, p, pl, stream)
                          : launch_qkv_cfg<64, 128, 2>(mx, mq, mk, mv, p, pl, stream);
  }
  if (pl.bn == 128)
    return pl.xrows == 64 ? launch_qkv_cfg<128, 64, 1>(mx, mq, mk, mv, p, pl, stream)
                          : launch_qkv_cfg<128, 128, 1>(mx, mq, mk, mv, p, pl, stream);
  return pl.xrows == 64 ? launch_qkv_cfg<64, 64, 1>(mx, mq, mk, mv, p, pl, stream)
                        : launch_qkv_cfg<64, 128, 1>(mx, mq, mk, mv, p, pl, stream);
}

}  // namespace
}  // namespace fdllm

extern "C" {

int fdllm_qkv_set_plan(int32_t impl, int32_t bn, int32_t splits, int32_t ksub, int32_t pair) {
  if (impl < -1 || impl > 1 || (bn != 0 && bn != 64 && bn != 128) || splits < 0 ||
      (ksub != 0 && ksub != 1 && ksub != 2) || pair < -1 || pair > 1)
    return FDLLM_ERR_ARG;
  fdllm::QkvOverride& o = fdllm::qkv_override();
  o.impl = impl;
  o.bn = bn;
  o.splits = splits < 1 ? 1 : splits;
  o.ksub = ksub;
  o.pair = pair;
  return FDLLM_OK;
}

size_t fdllm_qkv_workspace_bytes(int32_t n_rows, int32_t d_model, int32_t n_heads) {
  if (n_rows <= 0 || n_heads <= 0 || d_model != n_heads * 128) return 256;
  if (fdllm::qkv_use_sk(n_rows)) return fdllm::qkv_sk_ws_bytes(n_rows, d_model);
  return fdllm::qkv_ws_bytes(fdllm::plan_qkv(n_rows, d_model, n_heads));
}

int fdllm_qkv_rope_cache(const void* xn, const void* wq, const void* wk, const void* wv, const int64_t* pos,
                         const float* rope_sin, const float* rope_cos, void* q_out, void* k_cache, void* v_cache,
                         int32_t n_rows, int32_t d_model, int32_t n_heads, int64_t n_slots, void* workspace,
                         size_t workspace_bytes, cudaStream_t stream) {
  if (fdllm::qkv_use_sk(n_rows))
    return fdllm::launch_qkv_sk(xn, wq, wk, wv, pos, rope_sin, rope_cos, q_out, k_cache, v_cache, n_rows, d_model,
                                n_heads, n_slots, workspace, workspace_bytes, 1, stream);
  return fdllm::launch_qkv(xn, wq, wk, wv, pos, rope_sin, rope_cos, q_out, k_cache, v_cache, n_rows, d_model,
                           n_heads, n_slots, workspace, workspace_bytes, 1, stream);
}

int fdllm_verify_qkv(const void* xn, const void* wq, const void* wk, const void* wv, const int64_t* pos,
                     const float* rope_sin, const float* rope_cos, void* q_out, void* k_out, void* v_out,
                     int32_t n_rows, int32_t d_model, int32_t n_heads, int64_t n_slots, void* workspace,
                     size_t workspace_bytes, cudaStream_t stream) {
  if (fdllm::qkv_use_sk(n_rows))
    return fdllm::launch_qkv_sk(xn, wq, wk, wv, pos, rope_sin, rope_cos, q_out, k_out, v_out, n_rows, d_model,
                                n_heads, n_slots, workspace, workspace_bytes, 0, stream);
  return fdllm::launch_qkv(xn, wq, wk, wv, pos, rope_sin, rope_cos, q_out, k_out, v_out, n_rows, d_model,
                           n_heads, n_slots, workspace, workspace_bytes, 0, stream);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Entry point for callers that cannot allocate device memory.
//
// Some embedders drive this kernel from code that owns no device allocator:
// a host runtime whose memory is handed out by another component, a plugin
// loaded into a process that forbids cudaMalloc after start-up (to keep its
// pool fixed), or a caller inside a region that must not allocate.  They
// still pass the inputs and outputs, but not the split-K scratch
// (fdllm_qkv_rope_cache's `workspace`).  This variant takes that scratch from
// a fixed array compiled into the library instead.
//
//  * The array is kQkvNoAllocScratchBytes (24 MiB) of global memory on every
//    GPU that loads the library, held until the process exits.
//  * Requests whose scratch would exceed it are refused with
//    FDLLM_ERR_SCRATCH_LIMIT before anything is launched.  For LLaDA-8B
//    (d_model 4096) the stream-K GEMM, the default at every row count,
//    needs at most its flags plus one 128 KB partial per CTA (about 19 MB)
//    and fits; the earlier kernels' requested K splits above 128 rows do not.
//  * The first call on a device resolves the array's device address
//    (cudaGetSymbolAddress, with that device current); make that first call
//    before any stream capture.
//  * All calls share the array: its counter / flag region (split-K tile
//    counters, CTA-pair handoff flags) is zeroed on entry of every call that
//    uses the array, so a call that ended on a device error leaves nothing
//    behind for the next one; calls that overlap on the GPU (other streams,
//    other threads) race on it -- serialise them.
//  * No cudaMalloc / cudaFree or other allocating routine is called.
// ---------------------------------------------------------------------------
namespace {

constexpr size_t kQkvNoAllocScratchBytes = size_t(24) << 20;
static __device__ __align__(256) uint8_t g_qkv_noalloc_scratch[kQkvNoAllocScratchBytes];

void* qkv_noalloc_scratch() {
  static void* addr[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_qkv_noalloc_scratch) != cudaSuccess || p == nullptr) return nullptr;
    addr[dev] = p;
  }
  return addr[dev];
}

}  // namespace

extern "C" int fdllm_qkv_rope_cache_noalloc(const void* xn, const void* wq, const void* wk, const void* wv,
                                            const int64_t* pos, const float* rope_sin, const float* rope_cos,
                                            void* q_out, void* k_cache, void* v_cache, int32_t n_rows,
                                            int32_t d_model, int32_t n_heads, int64_t n_slots, cudaStream_t stream) {
  using namespace fdllm;
  if (n_rows < 0 || n_heads <= 0 || d_model != n_heads * 128 || n_slots <= 0) return FDLLM_ERR_ARG;
  if (n_rows == 0) return FDLLM_OK;
  if (qkv_use_sk(n_rows)) {
    // stream-K kernel: flags, then one partial accumulator per CTA
    if (qkv_sk_ws_bytes(n_rows, d_model) > kQkvNoAllocScratchBytes) return FDLLM_ERR_SCRATCH_LIMIT;
    void* scratch = qkv_noalloc_scratch();
    if (scratch == nullptr) return FDLLM_ERR_CUDA;
    if (cudaMemsetAsync(scratch, 0, kQkvCounterBytes, stream) != cudaSuccess) return FDLLM_ERR_CUDA;
    return launch_qkv_sk(xn, wq, wk, wv, pos, rope_sin, rope_cos, q_out, k_cache, v_cache, n_rows, d_model,
                         n_heads, n_slots, scratch, kQkvNoAllocScratchBytes, 1, stream);
  }
  const QkvPlan pl = plan_qkv(n_rows, d_model, n_heads);
  if ((pl.splits > 1 || pl.pair) && qkv_ws_bytes(pl) > kQkvNoAllocScratchBytes) return FDLLM_ERR_SCRATCH_LIMIT;
  void* scratch = qkv_noalloc_scratch();
  if (scratch == nullptr) return FDLLM_ERR_CUDA;
  // The counter / flag region at the front of the array is zeroed before
  // every call that uses the array: a call that ended on a device error may
  // have left split-K tile counters or CTA-pair handoff flags set, and this
  // caller has no other way to clear them.
  if ((pl.splits > 1 || pl.pair) && cudaMemsetAsync(scratch, 0, kQkvCounterBytes, stream) != cudaSuccess)
    return FDLLM_ERR_CUDA;
  return launch_qkv(xn, wq, wk, wv, pos, rope_sin, rope_cos, q_out, k_cache, v_cache, n_rows, d_model, n_heads,
                    n_slots, scratch, kQkvNoAllocScratchBytes, 1, stream);
}
