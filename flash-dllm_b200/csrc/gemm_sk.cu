// Persistent stream-K GEMM on tcgen05 tensor cores with fused epilogues:
//
//   C[rows, cols] = A[rows, K] * B[cols, K]^T      (bf16 in, fp32 accumulate)
//
// and, instead of storing C, one of
//   kEpiQkv    RoPE on the Q and K columns with the row's slot sin/cos, Q to
//              its row, K and V to cache row pos[r] (or row-indexed), where
//              B = [W_q; W_k; W_v] is given as three tensors
//              (ref llada/flash_cache_triton.py:15-100, 255-338);
//   kEpiStore  out = bf16(C (+ residual)) (ref :618-627, 634-636: attn_out,
//              ff_out and their residual adds; the LM head);
//   kEpiSwiglu B = [W_gate; W_up] stacked (2H rows): out[:, j] =
//              bf16(bf16(silu(bf16(gate_j))) * bf16(up_j)), so the gate / up
//              activations never reach HBM (ref :628-633).
//
// Work decomposition.  A tile is 128 rows x BN columns (BN = 128 or 256
// UMMA columns).  The CTAs form one group per 128-row m-tile; each group
// covers the (column tile, k-block) space of its m-tile, one contiguous range
// per CTA (stream-K), so every SM streams the same number of k-blocks
// whatever the tile count.  CTA j of every group has the same range, so the
// groups read each weight k-block at about the same time: it comes from
// DRAM once and from L2 for the other m-tiles.  At 64 rows the kernel is
// bound by reading the weights once from HBM, at 512 rows by the tensor
// cores.  (More m-tiles than SMs: one group, m-tiles innermost.)
//
// A range starts inside a tile ("tail piece": that tile's last k-blocks),
// runs over whole tiles and ends inside a tile ("head piece": its first
// k-blocks).  Tail pieces are always a CTA's first segment: the CTA stores
// its fp32 partial accumulator to its slot of the workspace and publishes it
// with a release flag.  The CTA holding a tile's head piece (its last
// segment) is the tile's owner: it waits for the flags of the CTAs after it
// whose ranges start inside the tile (they did those k-blocks first, so the
// wait is normally already over), adds their partials in CTA order -- a fixed
// order, so results do not depend on timing -- runs the epilogue and clears
// the flags for the next call.  Every CTA of the grid is resident at once
// (grid <= SMs, one CTA per SM), and every wait is bounded.
//
// Warp roles (192 threads): warp 0 TMA producer into a ring of KSUB x 64-K
// stages (128-byte swizzle), warp 1 TMEM owner and single-thread MMA issuer
// (M = 128, N = BN) into one of two TMEM accumulators (segments alternate),
// warps 2-5 the epilogue (thread = TMEM lane = tile row), which overlaps the
// next segment's MMAs.
#include "common.cuh"
#include "internal.h"

namespace fdllm {

constexpr int kGBM = 128;
constexpr int kGBK = 64;
constexpr int kGThreads = 192;
constexpr int kGemmKernelId = 7;
constexpr int kGRingBytes = 192 * 1024;
constexpr size_t kGFlagBytes = 4096;  // one int32 flag per CTA (grid <= 1024)

enum GemmEpi { kEpiQkv = 0, kEpiStore = 1, kEpiSwiglu = 2 };

template <int BN, int XROWS, int KSUB>
struct GCfg {
  static constexpr int kASub = XROWS * kGBK * 2;  // MMA reads 128 rows; rows >= XROWS are not used
  static constexpr int kBSub = BN * kGBK * 2;
  static constexpr int kABytes = KSUB * kASub;
  static constexpr int kStageBytes = KSUB * (kASub + kBSub);
  static constexpr int kStages = kGRingBytes / kStageBytes;
  static constexpr int kBarOffset = kStages * kStageBytes;
  static constexpr int kSmem = 1024 + kBarOffset + 256;
  static constexpr int kTmemCols = 2 * BN;
  static_assert(kStages >= 2, "ring depth");
  static_assert(kSmem <= 227 * 1024, "shared memory");
};

struct GemmParams {
  int32_t groups;    // CTA groups (one per m-tile, or 1)
  int32_t n_rows;
  int32_t n_cols;    // output columns of C (QKV: 3 d; store: N; swiglu: 2 H)
  int32_t m_tiles;
  int32_t n_tiles;
  int32_t kbt;       // k-blocks (KSUB x 64) per tile
  int32_t iters;     // iterations per group: n_tiles * kbt (x m_tiles with one group)
  int32_t epi;
  int32_t d_model;   // QKV: columns per projection
  int32_t hidden;    // swiglu: H (first up row of the stacked weight)
  int32_t kv_by_slot;
  int64_t n_slots;
  int64_t ld_out;
  int64_t ld_res;
  __nv_bfloat16* out0;  // QKV: q; store / swiglu: out
  __nv_bfloat16* out1;  // QKV: k
  __nv_bfloat16* out2;  // QKV: v
  const __nv_bfloat16* res;
  const int64_t* pos;
  const float* sin;
  const float* cos;
  float* partials;   // [grid][BN / 4][128][4] fp32
  int32_t* flags;    // [grid]
  int32_t* status;
};

struct GSeg {
  int tile, k0, k1;
};

__device__ __forceinline__ int g_lo(int cta, int grid, int iters) {
  return static_cast<int>(static_cast<long long>(cta) * iters / grid);
}

// next segment of the range [i, hi): the k-blocks of one tile
__device__ __forceinline__ bool g_next(int& i, int hi, int kbt, GSeg& s) {
  if (i >= hi) return false;
  s.tile = i / kbt;
  s.k0 = i % kbt;
  s.k1 = s.k0 + (hi - i) < kbt ? s.k0 + (hi - i) : kbt;
  i += s.k1 - s.k0;
  return true;
}

// 32 accumulator columns [col, col + 32) of this thread's row, plus the
// partial sums of contributor CTAs [q0, q1) in CTA order.
template <int BN>
__device__ __forceinline__ void g_chunk(uint32_t t_row, int col, const GemmParams& p, int q0, int q1, int r_tile,
                                        float (&v)[32]) {
  __syncwarp();
  tmem_ld_32x32b_x32(t_row + col, v);
  for (int q = q0; q < q1; ++q) {
    const float4* part = reinterpret_cast<const float4*>(p.partials) + static_cast<size_t>(q) * (kGBM * BN / 4);
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
      const float4 x = __ldcg(part + ((col + j) >> 2) * kGBM + r_tile);
      v[j] += x.x;
      v[j + 1] += x.y;
      v[j + 2] += x.z;
      v[j + 3] += x.w;
    }
  }
}

__device__ __forceinline__ void g_store32(__nv_bfloat16* dst, const float (&v)[32]) {
#pragma unroll
  for (int i = 0; i < 32; i += 8) {
    uint4 u;
    u.x = pack_bf16x2(v[i], v[i + 1]);
    u.y = pack_bf16x2(v[i + 2], v[i + 3]);
    u.z = pack_bf16x2(v[i + 4], v[i + 5]);
    u.w = pack_bf16x2(v[i + 6], v[i + 7]);
    *reinterpret_cast<uint4*>(dst + i) = u;
  }
}

__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

template <int BN, int XROWS, int KSUB, int EPI>
__global__ void __launch_bounds__(kGThreads, 1)
    gemm_sk_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b0,
                   const __grid_constant__ CUtensorMap map_b1, const __grid_constant__ CUtensorMap map_b2,
                   const GemmParams p) {
  using C = GCfg<BN, XROWS, KSUB>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kBarOffset);
  uint64_t* empty = full + C::kStages;
  uint64_t* acc_full = empty + C::kStages;  // [2] MMA -> epilogue
  uint64_t* acc_empty = acc_full + 2;       // [2] epilogue (4 warps) -> MMA
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int32_t* abort_flag = reinterpret_cast<volatile int32_t*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int cta = blockIdx.x;
  const int per_group = gridDim.x / p.groups;
  const int group = cta / per_group;  // the m-tile (one group: m-tiles innermost in the tile index)
  const int idx = cta % per_group;    // rank within the group
  const int lo = g_lo(idx, per_group, p.iters);
  const int hi = g_lo(idx + 1, per_group, p.iters);
  const int m_tiles_in = p.groups > 1 ? 1 : p.m_tiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 4);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_a);
    tma_prefetch_desc(&map_b0);
    if (EPI == kEpiQkv) {
      tma_prefetch_desc(&map_b1);
      tma_prefetch_desc(&map_b2);
    }
  }
  if (warp == 1) tmem_alloc(tmem_slot, C::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // A comes from the kernel before (programmatic launch)
  pdl_wait();
  pdl_launch_dependents();

  if (warp == 0) {
    // ------------------------------------------------------ TMA producer --
    if (lane == 0) {
      constexpr uint32_t kTx = static_cast<uint32_t>(C::kStageBytes);
      uint32_t g = 0;
      bool ok = true;
      int i = lo;
      GSeg sg;
      while (ok && g_next(i, hi, p.kbt, sg)) {
        const int m_tile = p.groups > 1 ? group : sg.tile % m_tiles_in, n_tile = sg.tile / m_tiles_in;
        const CUtensorMap* map_b = &map_b0;
        int b_row = n_tile * BN;
        if (EPI == kEpiQkv) {
          const int proj = b_row / p.d_model;
          map_b = proj == 0 ? &map_b0 : (proj == 1 ? &map_b1 : &map_b2);
          b_row -= proj * p.d_model;
        } else if (EPI == kEpiSwiglu) {
          b_row = n_tile * (BN / 2);
        }
        for (int kb = sg.k0; kb < sg.k1; ++kb, ++g) {
          const int s = g % C::kStages;
          const uint32_t ph = (g / C::kStages) & 1;
          if (g >= static_cast<uint32_t>(C::kStages) && !mbar_wait(&empty[s], ph ^ 1, p.status, kGemmKernelId)) {
            ok = false;
            break;
          }
          uint8_t* a0 = smem + s * C::kStageBytes;
          uint8_t* b0 = a0 + C::kABytes;
          mbar_arrive_expect_tx(&full[s], kTx);
#pragma unroll
          for (int sub = 0; sub < KSUB; ++sub) {
            const int kx = (kb * KSUB + sub) * kGBK;
            tma_load_2d(a0 + sub * C::kASub, &map_a, kx, m_tile * kGBM, &full[s]);
            uint8_t* b = b0 + sub * C::kBSub;
            if (EPI == kEpiSwiglu) {
              tma_load_2d(b, map_b, kx, b_row, &full[s]);
              tma_load_2d(b + (BN / 2) * 128, map_b, kx, p.hidden + b_row, &full[s]);
            } else {
              tma_load_2d(b, map_b, kx, b_row, &full[s]);
            }
          }
        }
      }
    }
  } else if (warp == 1) {
    // -------------------------------------------------------- MMA issuer --
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16(kGBM, BN);
      uint32_t g = 0;
      int seg = 0;
      bool ok = true;
      int i = lo;
      GSeg sg;
      while (ok && g_next(i, hi, p.kbt, sg)) {
        const int acc = seg & 1;
        if (seg >= 2 && !mbar_wait(&acc_empty[acc], ((seg >> 1) & 1) ^ 1, p.status, kGemmKernelId)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = sg.k0; kb < sg.k1; ++kb, ++g) {
          const int s = g % C::kStages;
          const uint32_t ph = (g / C::kStages) & 1;
          if (!mbar_wait(&full[s], ph, p.status, kGemmKernelId)) {
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
            for (int k = 0; k < kGBK / 16; ++k)
              umma_bf16(d_tmem, da + 2 * k, db + 2 * k, idesc, (kb > sg.k0 || sub > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&empty[s]);
        }
        if (!ok) break;
        umma_commit(&acc_full[acc]);
        ++seg;
      }
    }
  } else {
    // ---------------------------------------------------------- epilogue --
    const int quarter = warp & 3;
    const int r_tile = quarter * 32 + lane;
    const int ep_tid = threadIdx.x - 64;
    int seg = 0;
    int i = lo;
    GSeg sg;
    while (g_next(i, hi, p.kbt, sg)) {
      const int acc = seg & 1;
      const int m_tile = p.groups > 1 ? group : sg.tile % m_tiles_in, n_tile = sg.tile / m_tiles_in;
      const int row = m_tile * kGBM + r_tile;
      const bool row_ok = row < p.n_rows;
      const uint32_t t_row = tmem_base + acc * BN + (static_cast<uint32_t>(quarter * 32) << 16);
      // the QKV epilogue's slot and RoPE rows, fetched while the MMAs run
      int64_t slot = -1;
      if (EPI == kEpiQkv && sg.k0 == 0 && row_ok) {
        const int64_t s = p.pos[row];
        if (s < 0 || s >= p.n_slots) {
          report(p.status, FDLLM_ERR_INDEX, row, kGemmKernelId);
        } else {
          slot = s;
        }
      }
      // every epilogue thread reaches the named barriers (all waits are
      // bounded), so the decisions below are uniform over the 4 warps
      if (!mbar_wait(&acc_full[acc], (seg >> 1) & 1, p.status, kGemmKernelId)) *abort_flag = 1;
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (*abort_flag != 0) break;
      tc_fence_after();
      if (sg.k0 > 0) {
        // tail piece (this CTA's first segment): publish the partial sums,
        // [col / 4][row][4] fp32 so a warp's stores are 512 contiguous bytes
        float4* part = reinterpret_cast<float4*>(p.partials) + static_cast<size_t>(cta) * (kGBM * BN / 4);
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          float v[32];
          __syncwarp();
          tmem_ld_32x32b_x32(t_row + c, v);
#pragma unroll
          for (int j = 0; j < 32; j += 4)
            __stcg(part + ((c + j) >> 2) * kGBM + r_tile, make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]));
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[acc]);
        __threadfence();
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (ep_tid == 0) st_release_gpu(p.flags + cta, 1);
        ++seg;
        continue;
      }
      // whole tile, or the owner's head piece: wait for the contributors
      int q_end = cta + 1;  // contributors: the next CTAs of the group
      if (sg.k1 < p.kbt) {
        const int t_end = (sg.tile + 1) * p.kbt;
        while (q_end - group * per_group < per_group && g_lo(q_end - group * per_group, per_group, p.iters) < t_end)
          ++q_end;
        bool ok = true;
        if (ep_tid == 0)
          for (int q = cta + 1; q < q_end && ok; ++q) ok = flag_wait_set(p.flags + q, p.status, kGemmKernelId);
        if (!ok) *abort_flag = 1;
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (*abort_flag != 0) break;
      }
      const int q0 = cta + 1;
      if (EPI == kEpiQkv) {
#pragma unroll 1
        for (int hh = 0; hh < BN / 128; ++hh) {
          const int n0 = n_tile * BN + hh * 128;
          const int proj = n0 / p.d_model;
          const int hcol = n0 - proj * p.d_model;  // first column of the head in its projection
          __nv_bfloat16* dst = nullptr;
          if (slot >= 0) {
            const int64_t orow = (proj > 0 && p.kv_by_slot) ? slot : static_cast<int64_t>(row);
            dst = (proj == 0 ? p.out0 : (proj == 1 ? p.out1 : p.out2)) + orow * p.d_model + hcol;
          }
#pragma unroll 1
          for (int ch = 0; ch < 2; ++ch) {
            float a[32], b[32];
            g_chunk<BN>(t_row, hh * 128 + ch * 32, p, q0, q_end, r_tile, a);
            g_chunk<BN>(t_row, hh * 128 + 64 + ch * 32, p, q0, q_end, r_tile, b);
            if (dst == nullptr) continue;
            if (proj < 2) {
              const float* srow = p.sin + slot * 128 + ch * 32;
              const float* crow = p.cos + slot * 128 + ch * 32;
#pragma unroll
              for (int j = 0; j < 32; j += 4) {
                const float4 s1 = __ldg(reinterpret_cast<const float4*>(srow + j));
                const float4 s2 = __ldg(reinterpret_cast<const float4*>(srow + 64 + j));
                const float4 c1 = __ldg(reinterpret_cast<const float4*>(crow + j));
                const float4 c2 = __ldg(reinterpret_cast<const float4*>(crow + 64 + j));
                const float sa[4] = {s1.x, s1.y, s1.z, s1.w}, sb[4] = {s2.x, s2.y, s2.z, s2.w};
                const float ca[4] = {c1.x, c1.y, c1.z, c1.w}, cb[4] = {c2.x, c2.y, c2.z, c2.w};
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                  const float x1 = a[j + k], x2 = b[j + k];
                  a[j + k] = x1 * ca[k] - x2 * sa[k];
                  b[j + k] = x2 * cb[k] + x1 * sb[k];
                }
              }
            }
            g_store32(dst + ch * 32, a);
            g_store32(dst + 64 + ch * 32, b);
          }
        }
      } else if (EPI == kEpiStore) {
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          const int col = n_tile * BN + c;
          if (col >= p.n_cols) break;  // uniform; n_cols is a multiple of 32
          float v[32];
          g_chunk<BN>(t_row, c, p, q0, q_end, r_tile, v);
          if (!row_ok) continue;
          if (p.res != nullptr) {
            const __nv_bfloat16* rrow = p.res + static_cast<int64_t>(row) * p.ld_res + col;
#pragma unroll
            for (int j = 0; j < 32; j += 8) {
              const uint4 u = __ldg(reinterpret_cast<const uint4*>(rrow + j));
              const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[k]));
                v[j + 2 * k] += f.x;
                v[j + 2 * k + 1] += f.y;
              }
            }
          }
          g_store32(p.out0 + static_cast<int64_t>(row) * p.ld_out + col, v);
        }
      } else {
        // SwiGLU: UMMA columns [0, BN/2) are gate, [BN/2, BN) the matching up
#pragma unroll 1
        for (int c = 0; c < BN / 2; c += 32) {
          float gv[32], uv[32];
          g_chunk<BN>(t_row, c, p, q0, q_end, r_tile, gv);
          g_chunk<BN>(t_row, BN / 2 + c, p, q0, q_end, r_tile, uv);
          if (!row_ok) continue;
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const float gb = bf16_round(gv[j]);
            const float s = bf16_round(gb / (1.f + expf(-gb)));
            gv[j] = s * bf16_round(uv[j]);
          }
          g_store32(p.out0 + static_cast<int64_t>(row) * p.ld_out + n_tile * (BN / 2) + c, gv);
        }
      }
      // every column of this accumulator has been read
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[acc]);
      if (q_end > q0) {
        // every epilogue thread has read the partials: clear their flags
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (ep_tid == 0)
          for (int q = q0; q < q_end; ++q) p.flags[q] = 0;
      }
      ++seg;
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

struct GemmPlan {
  int bn, xrows, ksub, grid, groups;
  int m_tiles, n_tiles, kbt, iters;
};

// Plan overrides for tuning and tests (fdllm_gemm_set_plan): 0 = automatic.
struct GemmOverride {
  int bn, ksub, grid;
};
GemmOverride& gemm_override() {
  static GemmOverride o{env_int("FDLLM_GEMM_BN", 0), env_int("FDLLM_GEMM_KSUB", 0), env_int("FDLLM_GEMM_GRID", 0)};
  return o;
}

// Tile width: 128 columns up to 128 rows (the kernel streams weights from
// HBM; narrower tiles give more tiles, so fewer stream-K pieces per tile),
// 256 above (the kernel is bound by operand ingress per SM: a 128 x 256 tile
// moves 48 KB per 64-K step for 4.2 MFLOP, a 128 x 128 one 32 KB for 2.1).
GemmPlan plan_gemm(int epi, int32_t n_rows, int32_t n_cols, int32_t k_dim, int32_t d_model) {
  GemmPlan pl{};
  const GemmOverride& ov = gemm_override();
  pl.xrows = n_rows <= 64 ? 64 : 128;
  int bn = ov.bn == 128 || ov.bn == 256 ? ov.bn : (n_rows <= 128 ? 128 : 256);
  if (epi == kEpiQkv && d_model % bn != 0) bn = 128;
  pl.bn = bn;
  // two 64-K boxes per stage measured faster at every shape (256 B of every
  // weight row per request): 512 rows 51.7 vs 68.6 us (BN 256), 64 rows
  // 30.2 vs 31.1 us (BN 128)
  int ksub = ov.ksub == 1 || ov.ksub == 2 ? ov.ksub : 2;
  if (k_dim % (kGBK * ksub) != 0) ksub = 1;
  pl.ksub = ksub;
  pl.m_tiles = (n_rows + kGBM - 1) / kGBM;
  const int out_per_tile = epi == kEpiSwiglu ? bn / 2 : bn;
  const int out_cols = epi == kEpiSwiglu ? n_cols / 2 : n_cols;
  pl.n_tiles = (out_cols + out_per_tile - 1) / out_per_tile;
  pl.kbt = k_dim / (kGBK * ksub);
  // every CTA must be resident at once (owners wait for contributors), so
  // the grid never exceeds the SM count (one CTA per SM)
  int grid = sm_count();
  if (ov.grid > 0 && ov.grid < grid) grid = ov.grid;
  if (grid > 1024) grid = 1024;
  pl.groups = pl.m_tiles <= grid ? pl.m_tiles : 1;
  const long long iters = static_cast<long long>(pl.groups > 1 ? 1 : pl.m_tiles) * pl.n_tiles * pl.kbt;
  pl.iters = iters > (1ll << 30) ? -1 : static_cast<int>(iters);
  int per_group = grid / pl.groups;
  if (pl.iters > 0 && per_group > pl.iters) per_group = pl.iters;
  pl.grid = per_group * pl.groups;
  return pl;
}

size_t gemm_ws_bytes(const GemmPlan& pl) {
  return kGFlagBytes + static_cast<size_t>(pl.grid) * kGBM * pl.bn * sizeof(float);
}

template <int BN, int XROWS, int KSUB, int EPI>
int launch_gemm_cfg(const CUtensorMap& ma, const CUtensorMap& mb0, const CUtensorMap& mb1, const CUtensorMap& mb2,
                    const GemmParams& p, int grid, cudaStream_t stream) {
  using C = GCfg<BN, XROWS, KSUB>;
  static bool attr_set[64] = {false};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return FDLLM_ERR_CUDA;
  if (!attr_set[dev]) {
    if (cudaFuncSetAttribute(gemm_sk_kernel<BN, XROWS, KSUB, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             C::kSmem) != cudaSuccess)
      return FDLLM_ERR_CUDA;
    attr_set[dev] = true;
  }
  if (launch_ex(gemm_sk_kernel<BN, XROWS, KSUB, EPI>, dim3(grid), dim3(kGThreads), C::kSmem, stream, 1,
                pdl_enabled(), ma, mb0, mb1, mb2, p) != cudaSuccess)
    return FDLLM_ERR_CUDA;
  return cudaPeekAtLastError() == cudaSuccess ? FDLLM_OK : FDLLM_ERR_CUDA;
}

template <int EPI>
int dispatch_gemm(const GemmPlan& pl, const CUtensorMap& ma, const CUtensorMap& mb0, const CUtensorMap& mb1,
                  const CUtensorMap& mb2, const GemmParams& p, cudaStream_t stream) {
  if (pl.bn == 256) {
    if (pl.xrows == 64)
      return pl.ksub == 2 ? launch_gemm_cfg<256, 64, 2, EPI>(ma, mb0, mb1, mb2, p, pl.grid, stream)
                          : launch_gemm_cfg<256, 64, 1, EPI>(ma, mb0, mb1, mb2, p, pl.grid, stream);
    return launch_gemm_cfg<256, 128, 1, EPI>(ma, mb0, mb1, mb2, p, pl.grid, stream);
  }
  if (pl.xrows == 64)
    return pl.ksub == 2 ? launch_gemm_cfg<128, 64, 2, EPI>(ma, mb0, mb1, mb2, p, pl.grid, stream)
                        : launch_gemm_cfg<128, 64, 1, EPI>(ma, mb0, mb1, mb2, p, pl.grid, stream);
  return pl.ksub == 2 ? launch_gemm_cfg<128, 128, 2, EPI>(ma, mb0, mb1, mb2, p, pl.grid, stream)
                      : launch_gemm_cfg<128, 128, 1, EPI>(ma, mb0, mb1, mb2, p, pl.grid, stream);
}

// Shared set-up: plan, workspace split, tensor maps of A and of the weights.
int run_gemm(int epi, const void* a, int64_t lda, const void* const* w, int n_w, int64_t w_rows, int32_t n_rows,
             int32_t n_cols, int32_t k_dim, GemmParams& p, void* workspace, size_t workspace_bytes,
             cudaStream_t stream) {
  const GemmPlan pl = plan_gemm(epi, n_rows, n_cols, k_dim, p.d_model);
  if (pl.iters <= 0) return FDLLM_ERR_ARG;
  if (workspace == nullptr || workspace_bytes < gemm_ws_bytes(pl) || !aligned16(workspace))
    return FDLLM_ERR_WORKSPACE;
  p.groups = pl.groups;
  p.n_rows = n_rows;
  p.n_cols = n_cols;
  p.m_tiles = pl.m_tiles;
  p.n_tiles = pl.n_tiles;
  p.kbt = pl.kbt;
  p.iters = pl.iters;
  p.epi = epi;
  p.flags = static_cast<int32_t*>(workspace);
  p.partials = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + kGFlagBytes);
  p.status = status_ptr();
  CUtensorMap ma, mb[3];
  int rc;
  if ((rc = make_tmap_bf16_sw128(&ma, a, n_rows, k_dim, lda, pl.xrows)) != FDLLM_OK) return rc;
  const uint32_t box = epi == kEpiSwiglu ? pl.bn / 2 : pl.bn;
  for (int i = 0; i < n_w; ++i)
    if ((rc = make_tmap_bf16_sw128(&mb[i], w[i], w_rows, k_dim, k_dim, box)) != FDLLM_OK) return rc;
  for (int i = n_w; i < 3; ++i) mb[i] = mb[0];
  if (epi == kEpiQkv) return dispatch_gemm<kEpiQkv>(pl, ma, mb[0], mb[1], mb[2], p, stream);
  if (epi == kEpiStore) return dispatch_gemm<kEpiStore>(pl, ma, mb[0], mb[1], mb[2], p, stream);
  return dispatch_gemm<kEpiSwiglu>(pl, ma, mb[0], mb[1], mb[2], p, stream);
}

}  // namespace

// QKV through the stream-K kernel (called by the QKV entry points).
int launch_qkv_sk(const void* xn, const void* wq, const void* wk, const void* wv, const int64_t* pos,
                  const float* rope_sin, const float* rope_cos, void* q_out, void* k_out, void* v_out, int32_t n_rows,
                  int32_t d_model, int32_t n_heads, int64_t n_slots, void* workspace, size_t workspace_bytes,
                  int kv_by_slot, cudaStream_t stream) {
  if (n_rows < 0 || n_heads <= 0 || d_model != n_heads * 128 || n_slots <= 0 || d_model % kGBK != 0)
    return FDLLM_ERR_ARG;
  if (n_rows == 0) return FDLLM_OK;
  const void* ptrs[] = {xn, wq, wk, wv, pos, rope_sin, rope_cos, q_out, k_out, v_out};
  for (const void* x : ptrs)
    if (x == nullptr || !aligned16(x)) return FDLLM_ERR_ARG;
  GemmParams p{};
  p.d_model = d_model;
  p.kv_by_slot = kv_by_slot;
  p.n_slots = n_slots;
  p.out0 = static_cast<__nv_bfloat16*>(q_out);
  p.out1 = static_cast<__nv_bfloat16*>(k_out);
  p.out2 = static_cast<__nv_bfloat16*>(v_out);
  p.pos = pos;
  p.sin = rope_sin;
  p.cos = rope_cos;
  const void* w[3] = {wq, wk, wv};
  return run_gemm(kEpiQkv, xn, d_model, w, 3, d_model, n_rows, 3 * d_model, d_model, p, workspace, workspace_bytes,
                  stream);
}

size_t qkv_sk_ws_bytes(int32_t n_rows, int32_t d_model) {
  return gemm_ws_bytes(plan_gemm(kEpiQkv, n_rows, 3 * d_model, d_model, d_model));
}

}  // namespace fdllm

extern "C" {

int fdllm_gemm_set_plan(int32_t bn, int32_t ksub, int32_t grid) {
  if ((bn != 0 && bn != 128 && bn != 256) || (ksub != 0 && ksub != 1 && ksub != 2) || grid < 0 || grid > 1024)
    return FDLLM_ERR_ARG;
  fdllm::GemmOverride& o = fdllm::gemm_override();
  o.bn = bn;
  o.ksub = ksub;
  o.grid = grid;
  return FDLLM_OK;
}

size_t fdllm_gemm_workspace_bytes(int32_t n_rows, int32_t n_cols, int32_t k_dim, int32_t swiglu) {
  if (n_rows <= 0 || n_cols <= 0 || k_dim <= 0) return fdllm::kGFlagBytes;
  return fdllm::gemm_ws_bytes(
      fdllm::plan_gemm(swiglu ? fdllm::kEpiSwiglu : fdllm::kEpiStore, n_rows, n_cols, k_dim, 0));
}

int fdllm_gemm_bf16(const void* a, const void* w, void* out, const void* residual, int32_t n_rows, int32_t n_cols,
                    int32_t k_dim, int64_t ld_out, int64_t ld_res, void* workspace, size_t workspace_bytes,
                    cudaStream_t stream) {
  using namespace fdllm;
  if (n_rows < 0 || n_cols <= 0 || k_dim <= 0 || n_cols % 32 != 0 || k_dim % kGBK != 0 || ld_out < n_cols ||
      ld_out % 8 != 0 || (residual != nullptr && (ld_res < n_cols || ld_res % 8 != 0)))
    return FDLLM_ERR_ARG;
  if (n_rows == 0) return FDLLM_OK;
  if (a == nullptr || w == nullptr || out == nullptr || !aligned16(a) || !aligned16(w) || !aligned16(out) ||
      (residual != nullptr && !aligned16(residual)))
    return FDLLM_ERR_ARG;
  GemmParams p{};
  p.out0 = static_cast<__nv_bfloat16*>(out);
  p.res = static_cast<const __nv_bfloat16*>(residual);
  p.ld_out = ld_out;
  p.ld_res = ld_res;
  const void* ws[1] = {w};
  return run_gemm(kEpiStore, a, k_dim, ws, 1, n_cols, n_rows, n_cols, k_dim, p, workspace, workspace_bytes, stream);
}

int fdllm_gemm_swiglu(const void* a, const void* w_gate_up, void* out, int32_t n_rows, int32_t hidden, int32_t k_dim,
                      int64_t ld_out, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  using namespace fdllm;
  if (n_rows < 0 || hidden <= 0 || k_dim <= 0 || hidden % 128 != 0 || k_dim % kGBK != 0 || ld_out < hidden ||
      ld_out % 8 != 0)
    return FDLLM_ERR_ARG;
  if (n_rows == 0) return FDLLM_OK;
  if (a == nullptr || w_gate_up == nullptr || out == nullptr || !aligned16(a) || !aligned16(w_gate_up) ||
      !aligned16(out))
    return FDLLM_ERR_ARG;
  GemmParams p{};
  p.out0 = static_cast<__nv_bfloat16*>(out);
  p.ld_out = ld_out;
  p.hidden = hidden;
  const void* ws[1] = {w_gate_up};
  return run_gemm(kEpiSwiglu, a, k_dim, ws, 1, 2 * hidden, n_rows, 2 * hidden, k_dim, p, workspace, workspace_bytes,
                  stream);
}

}  // extern "C"
