// Decode bookkeeping kernels of the Flash-Cache / Flash-Verify loop
// (llada/generate.py), batched over sequences so one step needs one launch
// per decision instead of per-sequence host loops:
//
//   row_stats      fp64 softmax statistics of logit rows: max probability,
//                  first argmax, and optionally the probability of a given
//                  token (one CTA per row, two passes over the vocabulary).
//   window_accept  per sequence (one warp): zero probabilities past the
//                  predicted length, stable descending order of the masked
//                  window, keep = max(#(p >= threshold), min_keep), write the
//                  reordered window into full_pos, commit the kept tokens,
//                  record drafts and the EOS position.
//   verify_accept  per sequence: sequential fp64 cumprod of the drafts'
//                  mask-view probabilities, keep = #(cumprod >= gamma),
//                  commit the accepted drafts.
//   refresh_sort   per sequence (one CTA): stable ascending sort of the
//                  decoded slots by attention score, in place in full_pos
//                  (bitonic sort of unique (score, index) keys in smem).
//
// Integer outputs equal the reference's decisions whenever its torch.sort
// calls resolve ties in index order (the reference's sorts are not stable).
#include "common.cuh"
#include "internal.h"

namespace fdllm {

constexpr int kStatsThreads = 512;
constexpr int kDecodeKernelId = 5;
constexpr int kRefreshMax = 8192;

__device__ __forceinline__ float bf16_to_f(__nv_bfloat16 h) { return __bfloat162float(h); }

// ------------------------------------------------------------ row stats ----
// exp of every bf16 value in fp64, indexed by the bf16 bit pattern: for
// |x|, |m| <= 512, exp(x - m) = exp(x) * exp(-m), two correctly rounded
// factors and one rounded product (<= ~1.5 ulp, the order of the fp64
// summation's own rounding), one L1-resident load and one multiply instead of
// an fp64 exp per logit (the row pass was bound by fp64 exp throughput).
// Larger magnitudes take the fp64 exp.
__device__ double g_exp_bf16[65536];

__global__ void exp_table_kernel() {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < 65536) {
    const __nv_bfloat16 h = __ushort_as_bfloat16(static_cast<unsigned short>(i));
    const float x = __bfloat162float(h);
    g_exp_bf16[i] = fabsf(x) <= 512.f ? exp(static_cast<double>(x)) : 0.0;
  }
}

// |x| <= 512 for a bf16 bit pattern: exponent field below 2^9, finite
__device__ __forceinline__ bool small_bf16(unsigned short bits) { return (bits & 0x7f80u) < 0x4400u; }

__global__ void __launch_bounds__(kStatsThreads) row_stats_kernel(const __nv_bfloat16* __restrict__ logits,
                                                                  int64_t ld, int vocab,
                                                                  const int64_t* __restrict__ tokens,
                                                                  double* __restrict__ p_max,
                                                                  int64_t* __restrict__ argmax,
                                                                  double* __restrict__ p_tok) {
  const int64_t r = blockIdx.x;
  const __nv_bfloat16* row = logits + r * ld;
  __shared__ float s_max[kStatsThreads / 32];
  __shared__ int s_idx[kStatsThreads / 32];
  __shared__ double s_sum[kStatsThreads / 32];
  // 16-byte loads of 8 logits when the row allows it (the vocabulary and the
  // row stride multiples of 8, an aligned base), single logits for the rest
  const bool vec = (ld % 8 == 0) && ((reinterpret_cast<uintptr_t>(logits) & 15) == 0);
  const int nvec = vec ? vocab / 8 : 0;
  const uint4* rowv = reinterpret_cast<const uint4*>(row);
  float m = -INFINITY;
  int mi = INT32_MAX;
  // strictly greater: the first index wins within a thread (its indices increase)
#pragma unroll 4
  for (int i = threadIdx.x; i < nvec; i += kStatsThreads) {
    const uint4 u = __ldg(rowv + i);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __bfloat1622float2(h[e]);
      if (f.x > m) {
        m = f.x;
        mi = 8 * i + 2 * e;
      }
      if (f.y > m) {
        m = f.y;
        mi = 8 * i + 2 * e + 1;
      }
    }
  }
  for (int i = 8 * nvec + threadIdx.x; i < vocab; i += kStatsThreads) {
    const float v = bf16_to_f(row[i]);
    if (v > m) {
      m = v;
      mi = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float om = __shfl_xor_sync(0xffffffffu, m, o);
    const int oi = __shfl_xor_sync(0xffffffffu, mi, o);
    if (om > m || (om == m && oi < mi)) {
      m = om;
      mi = oi;
    }
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) {
    s_max[w] = m;
    s_idx[w] = mi;
  }
  __syncthreads();
  if (w == 0) {
    m = l < kStatsThreads / 32 ? s_max[l] : -INFINITY;
    mi = l < kStatsThreads / 32 ? s_idx[l] : INT32_MAX;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float om = __shfl_xor_sync(0xffffffffu, m, o);
      const int oi = __shfl_xor_sync(0xffffffffu, mi, o);
      if (om > m || (om == m && oi < mi)) {
        m = om;
        mi = oi;
      }
    }
    if (l == 0) {
      s_max[0] = m;
      s_idx[0] = mi;
    }
  }
  __syncthreads();
  const double md = static_cast<double>(s_max[0]);
  double sum = 0.0;
  const bool table = fabsf(s_max[0]) <= 512.f;
  const double em = table ? exp(-md) : 0.0;
#pragma unroll 2
  for (int i = threadIdx.x; i < nvec; i += kStatsThreads) {
    const uint4 u = __ldg(rowv + i);
    const unsigned short* b = reinterpret_cast<const unsigned short*>(&u);
    double part = 0.0;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      part += (table && small_bf16(b[e])) ? __ldg(g_exp_bf16 + b[e]) * em
                                          : exp(static_cast<double>(bf16_to_f(__ushort_as_bfloat16(b[e]))) - md);
    }
    sum += part;
  }
  for (int i = 8 * nvec + threadIdx.x; i < vocab; i += kStatsThreads) sum += exp(static_cast<double>(bf16_to_f(row[i])) - md);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  if (l == 0) s_sum[w] = sum;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int i = 0; i < kStatsThreads / 32; ++i) t += s_sum[i];
    p_max[r] = 1.0 / t;
    argmax[r] = s_idx[0];
    if (p_tok != nullptr) {
      const int64_t tk = tokens[r];
      p_tok[r] = (tk >= 0 && tk < vocab) ? exp(static_cast<double>(bf16_to_f(row[tk])) - md) / t : 0.0;
    }
  }
}

// -------------------------------------------------------- window accept ----
// seq_info int64 [B, 4]: (row offset into p/argmax/window, window length, num_decoded, predicted_length).
// eos_known int32 [B]: 1 when an EOS was decoded earlier (probabilities past the
// predicted length are zeroed).  Outputs per sequence: keep, length_num (window
// slots before the predicted length), eos_slot (largest committed slot holding
// eos_id, or -1).
struct AcceptArgs {
  const double* p;
  const int64_t* tok;
  const int64_t* window;   // flat slots of the masked window rows
  const int64_t* seq_info;
  const int32_t* eos_known;
  int64_t* full_pos;       // [B, lmax]
  int64_t* x;              // [B * lmax]
  int64_t* x_draft;        // [B * lmax] or null
  int32_t* keep_out;
  int32_t* length_out;
  int64_t* eos_out;
  int32_t* status;
  int64_t lmax;
  int64_t eos_id;
  double threshold;
  int32_t min_keep;
  int32_t batch;        // sequences in this call
  int64_t batch_slots;  // rows of full_pos; x and x_draft hold batch_slots * lmax tokens
};

constexpr int kAcceptMax = 256;

__global__ void __launch_bounds__(32) window_accept_kernel(const AcceptArgs a) {
  const int j = blockIdx.x;
  const int lane = threadIdx.x;
  const int64_t off = a.seq_info[4 * j + 0];
  const int n = static_cast<int>(a.seq_info[4 * j + 1]);
  const int64_t fp_at = a.seq_info[4 * j + 2];  // flat index of full_pos[slot, num_decoded]
  const int64_t pred = a.seq_info[4 * j + 3];
  const int64_t nd = fp_at >= 0 ? fp_at % a.lmax : -1;
  if (n <= 0 || n > kAcceptMax || nd < 0 || fp_at >= a.lmax * a.batch_slots || nd + n > a.lmax) {
    if (lane == 0) {
      if (n != 0) report(a.status, FDLLM_ERR_ARG, j, kDecodeKernelId);
      a.keep_out[j] = 0;
      a.length_out[j] = 0;
      a.eos_out[j] = -1;
    }
    return;
  }
  __shared__ double sp[kAcceptMax];
  __shared__ int64_t sslot[kAcceptMax], stok[kAcceptMax];
  __shared__ int64_t sorted_slot[kAcceptMax], sorted_tok[kAcceptMax];
  const bool zero_tail = a.eos_known[j] != 0;
  int above = 0, within = 0;
  for (int i = lane; i < n; i += 32) {
    double pv = a.p[off + i];
    const int64_t slot = a.window[off + i];
    const bool tail = slot >= pred;
    if (zero_tail && tail) pv = 0.0;
    sp[i] = pv;
    sslot[i] = slot;
    stok[i] = a.tok[off + i];
    above += pv >= a.threshold ? 1 : 0;
    within += (zero_tail && tail) ? 0 : 1;
    if (a.x_draft != nullptr && slot >= 0 && slot < a.lmax * a.batch_slots) a.x_draft[slot] = stok[i];
  }
  __syncwarp();
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    above += __shfl_xor_sync(0xffffffffu, above, o);
    within += __shfl_xor_sync(0xffffffffu, within, o);
  }
  // stable descending rank: #greater + #equal-before
  for (int i = lane; i < n; i += 32) {
    const double pi = sp[i];
    int rank = 0;
    for (int k = 0; k < n; ++k) {
      const double pk = sp[k];
      rank += (pk > pi || (pk == pi && k < i)) ? 1 : 0;
    }
    sorted_slot[rank] = sslot[i];
    sorted_tok[rank] = stok[i];
  }
  __syncwarp();
  const int keep = max(above, a.min_keep) < n ? max(above, a.min_keep) : n;
  int64_t* fp = a.full_pos + fp_at;
  int64_t eos = -1;
  for (int i = lane; i < n; i += 32) {
    const int64_t slot = sorted_slot[i];
    fp[i] = slot;
    if (i < keep && slot >= 0 && slot < a.lmax * a.batch_slots) {
      a.x[slot] = sorted_tok[i];
      if (sorted_tok[i] == a.eos_id) eos = max(eos, slot);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const int64_t oe = __shfl_xor_sync(0xffffffffu, eos, o);
    eos = oe > eos ? oe : eos;
  }
  if (lane == 0) {
    a.keep_out[j] = keep;
    a.length_out[j] = within;
    a.eos_out[j] = eos;
  }
}

// -------------------------------------------------------- verify accept ----
// seq_info int64 [B, 4]: (row offset into p/draft tokens, number of drafts S,
// num_decoded, predicted_length); eos_known as above; draft_slots are the flat
// slots of the draft rows (full_pos[j, nd:nd+S]).
struct VerifyArgs {
  const double* p;
  const int64_t* draft_tok;
  const int64_t* draft_slot;
  const int64_t* seq_info;
  const int32_t* eos_known;
  int64_t* x;
  int32_t* keep_out;
  int64_t* eos_out;
  int32_t* status;
  int64_t n_slots;
  int64_t eos_id;
  double gamma;
  int32_t batch;
};

__global__ void verify_accept_kernel(const VerifyArgs a) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= a.batch) return;
  const int64_t off = a.seq_info[4 * j + 0];
  const int s = static_cast<int>(a.seq_info[4 * j + 1]);
  const int64_t pred = a.seq_info[4 * j + 3];
  const bool zero_tail = a.eos_known[j] != 0;
  double cp = 1.0;
  int keep = 0;
  for (int i = 0; i < s; ++i) {  // sequential product: the order of torch.cumprod on the CPU
    double pv = a.p[off + i];
    if (zero_tail && a.draft_slot[off + i] >= pred) pv = 0.0;
    cp *= pv;
    keep += cp >= a.gamma ? 1 : 0;
  }
  int64_t eos = -1;
  for (int i = 0; i < keep; ++i) {
    const int64_t slot = a.draft_slot[off + i];
    if (slot < 0 || slot >= a.n_slots) {
      report(a.status, FDLLM_ERR_INDEX, j, kDecodeKernelId);
      continue;
    }
    a.x[slot] = a.draft_tok[off + i];
    if (a.draft_tok[off + i] == a.eos_id) eos = slot > eos ? slot : eos;
  }
  a.keep_out[j] = keep;
  a.eos_out[j] = eos;
}

// ---------------------------------------------------------- verify build ----
// The Flash-Verify forward's inputs of one step, built on the device from a
// few scalars per sequence (the reference builds them per sequence on the
// host, llada/generate.py:254-292).  seq int64 [n_seq, 8] = (slot row j,
// drafts s, num decoded nd, seqlen_k, predicted length, key offset, draft
// offset, unused).  Per sequence, 2 bm verify rows p: the t = 2 bm - 2 s
// decoded slots before nd (p < t), the s draft slots (t <= p < t + s, tokens
// from x_draft) and the same s slots again as the mask view (tokens from x);
// keys: its cache slots [0, nd - t) and [nd + s, seqlen_k); the (2 bm)^2 verify
// mask; the drafts' slots and logit rows; the attention's block row and the
// acceptance scan's (offset, s, 0, predicted length) row.
struct VBuildArgs {
  const int64_t* seq;
  const int64_t* full_pos;
  const int64_t* x;
  const int64_t* x_draft;
  int64_t* qpos;
  int64_t* xv;
  uint8_t* mask;
  int64_t* kpos;
  int64_t* dslot;
  int64_t* lidx;
  int32_t* vblocks;
  int64_t* info2;
  int32_t* status;
  int64_t n_slots;
  int64_t lmax;
  int32_t bm;
};

// (the reference's mask, generate.py:262-269: rows of the decoded slots do not
// see the drafts; drafts and their mask view see each other causally)
__device__ __forceinline__ uint8_t verify_mask_bit(int r, int c, int t, int s) {
  if (r < t) return (c >= t && c < t + s) ? 0 : 1;
  if (c < t || c >= t + 2 * s) return 1;
  const int rr = r - t, cc = c - t;
  if (rr < s) return cc < s ? (rr >= cc) : (rr < cc - s);
  return cc < s ? (rr - s > cc) : (rr - s <= cc - s);
}

__global__ void __launch_bounds__(256) verify_build_kernel(const VBuildArgs a) {
  const int k = blockIdx.x;
  const int64_t* q = a.seq + 8 * static_cast<int64_t>(k);
  const int64_t j = q[0], s = q[1], nd = q[2], sk = q[3], pred = q[4], koff = q[5], soff = q[6];
  const int R = 2 * a.bm;
  const int64_t t = R - 2 * s;
  const int64_t row0 = j * a.lmax;
  const int64_t base = row0 + nd;
  const int64_t len1 = nd - t > 0 ? nd - t : 0;
  const int64_t len2 = sk - nd - s > 0 ? sk - nd - s : 0;
  bool bad = s < 0 || t < 0;
  auto slot_at = [&](int64_t idx) -> int64_t {
    if (idx < row0 || idx >= row0 + a.lmax || idx >= a.n_slots) {
      bad = true;
      return 0;
    }
    return a.full_pos[idx];
  };
  for (int p = threadIdx.x; p < R && !(s < 0 || t < 0); p += blockDim.x) {
    const bool draft = p >= t && p < t + s;
    const int64_t off = p < t + s ? p - t : p - t - s;
    int64_t slot = slot_at(base + off);
    if (slot < 0 || slot >= a.n_slots) {
      bad = true;
      slot = 0;
    }
    a.qpos[static_cast<int64_t>(k) * R + p] = slot;
    a.xv[static_cast<int64_t>(k) * R + p] = draft ? a.x_draft[slot] : a.x[slot];
  }
  for (int e = threadIdx.x; e < R * R; e += blockDim.x)
    a.mask[(static_cast<int64_t>(k) * R + e / R) * R + e % R] =
        (s < 0 || t < 0) ? 1 : verify_mask_bit(e / R, e % R, static_cast<int>(t), static_cast<int>(s));
  for (int64_t i = threadIdx.x; i < s; i += blockDim.x) {
    a.dslot[soff + i] = slot_at(base + i);
    a.lidx[soff + i] = static_cast<int64_t>(k) * R + t + s + i;
  }
  for (int64_t n = threadIdx.x; n < len1 + len2; n += blockDim.x)
    a.kpos[koff + n] = slot_at(n < len1 ? row0 + n : base + s + (n - len1));
  if (threadIdx.x == 0) {
    a.vblocks[4 * k + 0] = static_cast<int32_t>(koff);
    a.vblocks[4 * k + 1] = static_cast<int32_t>(koff + len1 + len2);
    a.vblocks[4 * k + 2] = k * R;
    a.vblocks[4 * k + 3] = k * R + R;
    a.info2[4 * k + 0] = soff;
    a.info2[4 * k + 1] = s;
    a.info2[4 * k + 2] = 0;
    a.info2[4 * k + 3] = pred;
  }
  if (bad) report(a.status, FDLLM_ERR_INDEX, k, kDecodeKernelId);
}

// ----------------------------------------------------------- cache build ----
// The Flash-Cache forward's inputs of one step on the device (the reference's
// block tables and query lists, llada/generate.py:146-163, 439-465).  seq int64
// [n_seq, 16] = (slot row j, k_end, num decoded nd, predicted length, masked
// range start, masked count, tracked range 1 start, count, tracked range 2
// start, count, masked row offset, tracked row offset, masked tile offset,
// tracked tile offset, unused, unused); positions are indices into row j of
// full_pos.  Writes the sequence's query rows (slots and tokens: its masked
// rows among the first rows of the row space, its tracked rows after all
// masked ones), its block-table rows (seq, k_end, row begin, row end) in
// tiles of bm rows, and its window-acceptance row (masked row offset,
// masked count, flat index of nd, predicted length).
struct CBuildArgs {
  const int64_t* seq;
  const int64_t* full_pos;
  const int64_t* x;
  int64_t* tables;
  int64_t* qpos;
  int64_t* xq;
  int64_t* seq_info;
  int32_t* status;
  int64_t n_slots;
  int64_t lmax;
  int32_t bm;
};

__global__ void __launch_bounds__(256) cache_build_kernel(const CBuildArgs a) {
  const int k = blockIdx.x;
  const int64_t* q = a.seq + 16 * static_cast<int64_t>(k);
  const int64_t j = q[0], k_end = q[1], nd = q[2], pred = q[3];
  const int64_t ma = q[4], mn = q[5], t1a = q[6], t1n = q[7], t2a = q[8], t2n = q[9];
  const int64_t mo = q[10], to = q[11], mt = q[12], tt = q[13];
  const int64_t row0 = j * a.lmax, tn = t1n + t2n;
  bool bad = false;
  auto put = [&](int64_t row, int64_t pos) {
    int64_t slot = 0;
    if (pos < 0 || pos >= a.lmax || row0 + pos >= a.n_slots) {
      bad = true;
    } else {
      slot = a.full_pos[row0 + pos];
      if (slot < 0 || slot >= a.n_slots) {
        bad = true;
        slot = 0;
      }
    }
    a.qpos[row] = slot;
    a.xq[row] = a.x[slot];
  };
  for (int64_t i = threadIdx.x; i < mn; i += blockDim.x) put(mo + i, ma + i);
  for (int64_t i = threadIdx.x; i < tn; i += blockDim.x) put(to + i, i < t1n ? t1a + i : t2a + (i - t1n));
  for (int64_t u = threadIdx.x; u * a.bm < mn; u += blockDim.x) {
    int64_t* r = a.tables + 4 * (mt + u);
    r[0] = j;
    r[1] = k_end;
    r[2] = mo + u * a.bm;
    r[3] = mo + ((u + 1) * a.bm < mn ? (u + 1) * a.bm : mn);
  }
  for (int64_t u = threadIdx.x; u * a.bm < tn; u += blockDim.x) {
    int64_t* r = a.tables + 4 * (tt + u);
    r[0] = j;
    r[1] = k_end;
    r[2] = to + u * a.bm;
    r[3] = to + ((u + 1) * a.bm < tn ? (u + 1) * a.bm : tn);
  }
  if (threadIdx.x == 0) {
    a.seq_info[4 * k + 0] = mo;
    a.seq_info[4 * k + 1] = mn;
    a.seq_info[4 * k + 2] = row0 + nd;
    a.seq_info[4 * k + 3] = pred;
  }
  if (bad) report(a.status, FDLLM_ERR_INDEX, k, kDecodeKernelId);
}

// --------------------------------------------------------- refresh sort ----
// Orderable 32-bit image of a float for ascending order; -0 sorts as +0 and
// NaN after +inf (torch.sort's placement).
__device__ __forceinline__ uint32_t float_key(float f) {
  if (f != f) return 0xFFFFFFFFu;
  if (f == 0.f) f = 0.f;
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// counts int64 [B]: number of leading full_pos entries of each sequence to sort.
__global__ void __launch_bounds__(1024) refresh_sort_kernel(int64_t* __restrict__ full_pos, int64_t lmax,
                                                            const int64_t* __restrict__ counts,
                                                            const float* __restrict__ scores, int64_t n_slots,
                                                            int32_t* status) {
  extern __shared__ uint64_t keys[];
  const int j = blockIdx.x;
  const int n = static_cast<int>(counts[j]);
  if (n <= 1) return;
  if (n > kRefreshMax || n > lmax) {
    if (threadIdx.x == 0) report(status, FDLLM_ERR_ARG, j, kDecodeKernelId);
    return;
  }
  int64_t* fp = full_pos + static_cast<int64_t>(j) * lmax;
  int pow2 = 1;
  while (pow2 < n) pow2 <<= 1;
  for (int i = threadIdx.x; i < pow2; i += blockDim.x) {
    if (i < n) {
      const int64_t slot = fp[i];
      const float sc = (slot >= 0 && slot < n_slots) ? scores[slot] : INFINITY;
      keys[i] = (static_cast<uint64_t>(float_key(sc)) << 32) | static_cast<uint32_t>(i);
    } else {
      keys[i] = ~0ull;
    }
  }
  __syncthreads();
  for (int k = 2; k <= pow2; k <<= 1) {
    for (int jj = k >> 1; jj > 0; jj >>= 1) {
      for (int i = threadIdx.x; i < pow2; i += blockDim.x) {
        const int ixj = i ^ jj;
        if (ixj > i) {
          const uint64_t a = keys[i], b = keys[ixj];
          const bool up = (i & k) == 0;
          if ((a > b) == up) {
            keys[i] = b;
            keys[ixj] = a;
          }
        }
      }
      __syncthreads();
    }
  }
  // gather: new position i takes the slot that was at index (key & 0xffffffff)
  int64_t tmp[kRefreshMax / 1024];
  const int per = (n + blockDim.x - 1) / blockDim.x;  // <= 8 for n <= 8192
  for (int t = 0; t < per; ++t) {
    const int i = threadIdx.x + t * blockDim.x;
    tmp[t] = i < n ? fp[static_cast<uint32_t>(keys[i] & 0xFFFFFFFFull)] : 0;
  }
  __syncthreads();
  for (int t = 0; t < per; ++t) {
    const int i = threadIdx.x + t * blockDim.x;
    if (i < n) fp[i] = tmp[t];
  }
}

}  // namespace fdllm

extern "C" {

int fdllm_row_stats(const void* logits, int64_t ld, int32_t n_rows, int32_t vocab, const int64_t* tokens,
                    double* p_max, int64_t* argmax, double* p_tok, cudaStream_t stream) {
  if (n_rows < 0 || vocab <= 0 || ld < vocab || logits == nullptr || p_max == nullptr || argmax == nullptr ||
      (p_tok != nullptr && tokens == nullptr))
    return FDLLM_ERR_ARG;
  if (n_rows == 0) return FDLLM_OK;
  static bool table_ready[64] = {false};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return FDLLM_ERR_CUDA;
  if (!table_ready[dev]) {  // stream-ordered before the first row pass on this device
    fdllm::exp_table_kernel<<<256, 256, 0, stream>>>();
    if (cudaPeekAtLastError() != cudaSuccess) return FDLLM_ERR_CUDA;
    table_ready[dev] = true;
  }
  fdllm::row_stats_kernel<<<n_rows, fdllm::kStatsThreads, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(logits), ld, vocab, tokens, p_max, argmax, p_tok);
  return cudaPeekAtLastError() == cudaSuccess ? FDLLM_OK : FDLLM_ERR_CUDA;
}

int fdllm_window_accept(const double* p, const int64_t* tok, const int64_t* window, const int64_t* seq_info,
                        const int32_t* eos_known, int32_t batch, int64_t batch_slots, int64_t lmax, double threshold,
                        int32_t min_keep, int64_t eos_id, int64_t* full_pos, int64_t* x, int64_t* x_draft,
                        int32_t* keep_out, int32_t* length_out, int64_t* eos_out, cudaStream_t stream) {
  if (batch < 0 || lmax <= 0 || min_keep < 0 || batch_slots <= 0) return FDLLM_ERR_ARG;
  if (batch == 0) return FDLLM_OK;
  const void* ptrs[] = {p, tok, window, seq_info, eos_known, full_pos, x, keep_out, length_out, eos_out};
  for (const void* q : ptrs)
    if (q == nullptr) return FDLLM_ERR_ARG;
  fdllm::AcceptArgs a{p, tok, window, seq_info, eos_known, full_pos, x, x_draft, keep_out, length_out, eos_out,
                      fdllm::status_ptr(), lmax, eos_id, threshold, min_keep, batch, batch_slots};
  fdllm::window_accept_kernel<<<batch, 32, 0, stream>>>(a);
  return cudaPeekAtLastError() == cudaSuccess ? FDLLM_OK : FDLLM_ERR_CUDA;
}

int fdllm_verify_accept(const double* p, const int64_t* draft_tok, const int64_t* draft_slot,
                        const int64_t* seq_info, const int32_t* eos_known, int32_t batch, int64_t n_slots,
                        double gamma, int64_t eos_id, int64_t* x, int32_t* keep_out, int64_t* eos_out,
                        cudaStream_t stream) {
  if (batch < 0 || n_slots <= 0) return FDLLM_ERR_ARG;
  if (batch == 0) return FDLLM_OK;
  const void* ptrs[] = {seq_info, eos_known, x, keep_out, eos_out};
  for (const void* q : ptrs)
    if (q == nullptr) return FDLLM_ERR_ARG;
  fdllm::VerifyArgs a{p, draft_tok, draft_slot, seq_info, eos_known, x, keep_out, eos_out, fdllm::status_ptr(),
                      n_slots, eos_id, gamma, batch};
  fdllm::verify_accept_kernel<<<(batch + 127) / 128, 128, 0, stream>>>(a);
  return cudaPeekAtLastError() == cudaSuccess ? FDLLM_OK : FDLLM_ERR_CUDA;
}

int fdllm_verify_build(const int64_t* seq, int32_t n_seq, int32_t bm, int64_t lmax, int64_t n_slots,
                       const int64_t* full_pos, const int64_t* x, const int64_t* x_draft, int64_t* qpos, int64_t* xv,
                       uint8_t* mask, int64_t* kpos, int64_t* dslot, int64_t* lidx, int32_t* vblocks, int64_t* info2,
                       cudaStream_t stream) {
  if (n_seq < 0 || bm <= 0 || bm > 512 || lmax <= 0 || n_slots <= 0) return FDLLM_ERR_ARG;
  if (n_seq == 0) return FDLLM_OK;
  const void* ptrs[] = {seq, full_pos, x, x_draft, qpos, xv, mask, vblocks, info2};
  for (const void* q : ptrs)
    if (q == nullptr) return FDLLM_ERR_ARG;
  fdllm::VBuildArgs a{seq,  full_pos, x,     x_draft, qpos, xv, mask, kpos, dslot, lidx, vblocks, info2,
                      fdllm::status_ptr(), n_slots, lmax, bm};
  fdllm::verify_build_kernel<<<n_seq, 256, 0, stream>>>(a);
  return cudaPeekAtLastError() == cudaSuccess ? FDLLM_OK : FDLLM_ERR_CUDA;
}

int fdllm_cache_build(const int64_t* seq, int32_t n_seq, int32_t bm, int64_t lmax, int64_t n_slots,
                      const int64_t* full_pos, const int64_t* x, int64_t* tables, int64_t* qpos, int64_t* xq,
                      int64_t* seq_info, cudaStream_t stream) {
  if (n_seq < 0 || bm <= 0 || lmax <= 0 || n_slots <= 0) return FDLLM_ERR_ARG;
  if (n_seq == 0) return FDLLM_OK;
  const void* ptrs[] = {seq, full_pos, x, seq_info};
  for (const void* q : ptrs)
    if (q == nullptr) return FDLLM_ERR_ARG;
  fdllm::CBuildArgs a{seq, full_pos, x, tables, qpos, xq, seq_info, fdllm::status_ptr(), n_slots, lmax, bm};
  fdllm::cache_build_kernel<<<n_seq, 256, 0, stream>>>(a);
  return cudaPeekAtLastError() == cudaSuccess ? FDLLM_OK : FDLLM_ERR_CUDA;
}

int fdllm_refresh_sort(int64_t* full_pos, int32_t batch, int64_t lmax, const int64_t* counts, const float* scores,
                       int64_t n_slots, cudaStream_t stream) {
  if (batch < 0 || lmax <= 0 || full_pos == nullptr || counts == nullptr || scores == nullptr) return FDLLM_ERR_ARG;
  if (batch == 0) return FDLLM_OK;
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  const int smem = fdllm::kRefreshMax * sizeof(uint64_t);
  if (dev < 64 && !attr[dev]) {
    if (cudaFuncSetAttribute(fdllm::refresh_sort_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
        cudaSuccess)
      return FDLLM_ERR_CUDA;
    attr[dev] = true;
  }
  fdllm::refresh_sort_kernel<<<batch, 1024, smem, stream>>>(full_pos, lmax, counts, scores, n_slots,
                                                             fdllm::status_ptr());
  return cudaPeekAtLastError() == cudaSuccess ? FDLLM_OK : FDLLM_ERR_CUDA;
}

}  // extern "C"
