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
// counter for the next call.
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
};

// Units are spread round-robin over one CTA per SM.  Tiles are 128 columns
// (one head) wide and K is not split by default: at 64 and 128 rows (96
// tiles) whole-K tiles on 96 SMs measured faster than 64-wide tiles on all
// SMs (64 rows: 35.5 vs 39.6 us) and than 2-6 K splits, whose fp32 partials
// cost more than the balance gains (64 rows: 41.7-92 us).  FDLLM_QKV_BN /
// FDLLM_QKV_SPLITS / FDLLM_QKV_KSUB override the choices.
QkvPlan plan_qkv(int32_t n_rows, int32_t d_model, int32_t n_heads) {
  QkvPlan pl{};
  int ksub = env_int("FDLLM_QKV_KSUB", 0);
  if (ksub != 1 && ksub != 2) ksub = 2;
  if (d_model % (kQkvBK * ksub) != 0) ksub = 1;
  pl.ksub = ksub;
  const int kb_total = d_model / (kQkvBK * ksub);
  const int sms = sm_count();
  pl.m_tiles = (n_rows + kQkvBM - 1) / kQkvBM;
  pl.xrows = n_rows <= 64 ? 64 : 128;
  int bn = env_int("FDLLM_QKV_BN", 0);
  if (bn != 64 && bn != 128) bn = 128;
  pl.bn = bn;
  pl.n_tiles = 3 * n_heads * (128 / bn);
  const int tiles = pl.m_tiles * pl.n_tiles;
  int splits = env_int("FDLLM_QKV_SPLITS", 1);
  if (splits < 1) splits = 1;
  if (splits > kb_total) splits = kb_total;
  pl.kb_per_split = (kb_total + splits - 1) / splits;
  pl.splits = (kb_total + pl.kb_per_split - 1) / pl.kb_per_split;  // no empty splits
  pl.n_units = tiles * pl.splits;
  pl.grid = pl.n_units < sms ? pl.n_units : sms;
  return pl;
}

// Workspace layout: a fixed counter region (so counters never move between
// calls with different tile counts, and no call's partial sums land on another
// call's counters), then the split-K partials.
constexpr size_t kQkvCounterBytes = 4096;  // 1024 tiles (K splits are requested through FDLLM_QKV_SPLITS)

size_t qkv_ws_bytes(const QkvPlan& pl) {
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
  qkv_rope_kernel<BN, XROWS, KSUB><<<pl.grid, kQkvThreads, C::kSmem, stream>>>(mx, mq, mk, mv, p);
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
  if (pl.splits > 1 && (workspace == nullptr || workspace_bytes < qkv_ws_bytes(pl))) return FDLLM_ERR_WORKSPACE;
  CUtensorMap mx, mq, mk, mv;
  int rc;
  if ((rc = make_tmap_bf16_sw128(&mx, xn, n_rows, d_model, d_model, pl.xrows)) != FDLLM_OK) return rc;
  const uint32_t wbox = pl.bn == 128 ? 128 : pl.bn / 2;
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
  if (pl.splits > 1) {
    if (static_cast<size_t>(pl.m_tiles) * pl.n_tiles * sizeof(int32_t) > kQkvCounterBytes) return FDLLM_ERR_ARG;
    p.counters = static_cast<int32_t*>(workspace);
    p.partials = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + kQkvCounterBytes);
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

size_t fdllm_qkv_workspace_bytes(int32_t n_rows, int32_t d_model, int32_t n_heads) {
  if (n_rows <= 0 || n_heads <= 0 || d_model != n_heads * 128) return 256;
  return fdllm::qkv_ws_bytes(fdllm::plan_qkv(n_rows, d_model, n_heads));
}

int fdllm_qkv_rope_cache(const void* xn, const void* wq, const void* wk, const void* wv, const int64_t* pos,
                         const float* rope_sin, const float* rope_cos, void* q_out, void* k_cache, void* v_cache,
                         int32_t n_rows, int32_t d_model, int32_t n_heads, int64_t n_slots, void* workspace,
                         size_t workspace_bytes, cudaStream_t stream) {
  return fdllm::launch_qkv(xn, wq, wk, wv, pos, rope_sin, rope_cos, q_out, k_cache, v_cache, n_rows, d_model,
                           n_heads, n_slots, workspace, workspace_bytes, 1, stream);
}

int fdllm_verify_qkv(const void* xn, const void* wq, const void* wk, const void* wv, const int64_t* pos,
                     const float* rope_sin, const float* rope_cos, void* q_out, void* k_out, void* v_out,
                     int32_t n_rows, int32_t d_model, int32_t n_heads, int64_t n_slots, void* workspace,
                     size_t workspace_bytes, cudaStream_t stream) {
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
//  * Requests whose split-K scratch would exceed it are refused with
//    FDLLM_ERR_SCRATCH_LIMIT before anything is launched (for LLaDA-8B,
//    d_model 4096, that is any call of more than 128 query rows; calls that
//    need no split, such as 512 rows, use no scratch and are accepted).
//  * The first call on a device resolves the array's device address
//    (cudaGetSymbolAddress, with that device current); make that first call
//    before any stream capture.
//  * All calls share the array: the split counters are cleared at the start
//    of every call, and calls that overlap on the GPU (other streams, other
//    threads) race on it -- serialise them.
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
  const QkvPlan pl = plan_qkv(n_rows, d_model, n_heads);
  if (pl.splits > 1 && qkv_ws_bytes(pl) > kQkvNoAllocScratchBytes) return FDLLM_ERR_SCRATCH_LIMIT;
  void* scratch = qkv_noalloc_scratch();
  if (scratch == nullptr) return FDLLM_ERR_CUDA;
  if (pl.splits > 1 && cudaMemsetAsync(scratch, 0, kQkvCounterBytes, stream) != cudaSuccess) return FDLLM_ERR_CUDA;
  return launch_qkv(xn, wq, wk, wv, pos, rope_sin, rope_cos, q_out, k_cache, v_cache, n_rows, d_model, n_heads,
                    n_slots, scratch, kQkvNoAllocScratchBytes, 1, stream);
}
