// INT4 paged decode attention for sm_100a.
//
// Replaces the reference kernel _int4_paged_decode_attention
// (src/iris_kernel/fused_attention.py:11-220); semantics are those of
// torch_eager_int4_paged_decode_attention (src/iris_kernel/
// torch_eager_attention.py:154-239): for every sequence b and query head h,
// softmax(scale * q . k_l) weighted sum of v_l over the sequence's tokens,
// with k/v dequantised from the paged INT4 cache and query head h reading KV
// head h / (Hq/Hkv).
//
// Decomposition (split-KV, stream-K style).  The concatenation of all
// sequences' pages is cut into R equal ranges of whole pages; CTA (r, hb)
// walks range r for KV-head block hb.  A sequence that lies entirely inside
// one range is finished by that CTA; pieces of a sequence that straddles
// ranges leave (m, l, O) records that the combine kernel merges.  Work per
// CTA is therefore equal whatever the length distribution.
//
// CTA = HB consumer warps (one per KV head of the block) + 1 producer warp.
// The producer walks the page table and moves, per page and stage, each
// head's 16 x D/2-byte K and V tiles with a 3-D TMA tensor copy (swizzled so
// ldmatrix is conflict-free) and the page's K / V scale blocks with 1-D bulk
// copies, into an S-deep ring of shared-memory stages guarded by mbarriers.
//
// Consumer math per page and head (16 tokens):
//   S^T[tok][qh] = K[tok][:] . Q[qh][:]  as mma.m16n8k16 with M = tokens and
//     N = query heads (8 per n-tile).  K stays in biased integer form
//     (n + 1032 or 16 n + 1152 from a single LOP3 per half2) and each 32-dim
//     group has its own accumulator, seeded with minus the bias correction, so
//     the per-(token, group) scale is applied once in fp32 afterwards.
//   online softmax in the log2 domain, P rounded to fp16 and transposed into
//     the B operand with movmatrix; the V group scales multiply P (per token,
//     per group) rather than the 4x larger V tile.
//   O^T[dim][qh] += V^T[dim][tok] . P'^T[tok][qh] as mma.m16n8k16 with M =
//     head dims, from ldmatrix.trans fragments converted to exact fp16 ints.
// Head-dim permutations that make every 32-bit nibble word land on its MMA
// fragment slots are undone when Q is loaded and when O is stored.
#include <cstdio>
#include <cstdlib>
#include <map>
#include <mutex>
#include <tuple>
#include <utility>

#include "common.cuh"

namespace iris {

static thread_local char g_last_error[256] = "";

const char* record_cuda_error(cudaError_t e, const char* where) {
  snprintf(g_last_error, sizeof(g_last_error), "%s: %s (%s)", where, cudaGetErrorName(e), cudaGetErrorString(e));
  return g_last_error;
}

cudaError_t clear_stale_cuda_error() { return cudaGetLastError(); }

constexpr int kPage = 16;
constexpr int kMinPagesPerRange = 4;  // ranges hold at least this many pages ...
constexpr int kOnePageRanges = 48;    // ... but one page when the batch has at most this many
constexpr int kTwoPageRanges = 128;   // ... and two when it has at most this many

// Page ranges a batch of U pages is cut into (before the grid's cap).  Small
// batches get shorter ranges, so their CTAs wait for one or two copies
// instead of four in a row (batch-1 decode of 8 / 32 / 128 pages 10.4 / 10.4
// / 12.4 -> 8.2 / 8.9 / 10.4 us); from 256 pages up shorter ranges cost more
// in the combine than they save (256 pages after an L2 flush: 16.5 us at
// four, 18.3 at two; 1024 pages: 14.5 us at four, 16.5 at two).
__host__ __device__ __forceinline__ int64_t wanted_ranges(int64_t U) {
  if (U <= kOnePageRanges) return U;
  if (U <= kTwoPageRanges) return (U + 1) / 2;
  return (U + kMinPagesPerRange - 1) / kMinPagesPerRange;
}
#define kNegInf (-__int_as_float(0x7f800000))

struct DecodeParams {
  const __half* query;       // [B, Hq, D]
  const uint8_t* k_scale;    // [NP, 16, Hkv, D/32] fp16, as bytes
  const uint8_t* v_scale;
  const int32_t* block_table;
  int64_t bt_stride;
  const int32_t* seq_lens;
  void* out;                 // fp16 [B,Hq,D] or fp32 [B,Hq,D]
  float* out_lse;            // [B,Hq] (LSE mode)
  float* rec_o;              // [R, 2, Hq, D]
  float* rec_lse;            // [R, 2, Hq]
  const int32_t* prefix;     // [B+1] page prefix sums (written by the leader CTA for the combine)
  const int32_t* meta;       // [0] total pages U, [1] ranges in use (likewise)
  int32_t* err;
  int64_t num_pages;
  int32_t batch, hq, hkv, max_pages;
  int32_t hb;                // KV heads per CTA (= consumer warps)
  int32_t qpk;               // query heads per KV head
  int32_t stages;
  int32_t out_mode;
  int32_t ranges;            // page ranges launched (the decode grid's y extent)
  int32_t combine_lanes;     // lanes of the combine merging one output quad (1, 2, 4 or 8)
  float scale_log2;          // softmax_scale * log2(e)
};

template <int D>
struct DecCfg {
  static constexpr int kTileBytes = kPage * D / 2;  // one head's K (or V) tile of a page
  static constexpr int kGroups = D / 32;
  static constexpr int kScaleRowBytes = kGroups * 2;  // one (token, head) scale row
};

IRIS_DEV int64_t range_start(int64_t r, int64_t U, int64_t R) { return r * U / R; }
IRIS_DEV int64_t range_of_page(int64_t u, int64_t U, int64_t R) { return ((u + 1) * R - 1) / U; }

// ------------------------------------------------------------- planning
// Done by warp 0 of every decode CTA at start (no separate kernel): the total
// page count U of the batch, the number R of page ranges in use, and for this
// CTA's range r its first sequence and that sequence's first page.  The
// leader CTA (0, 0) also validates the lengths and writes the page prefix
// sums and (U, R) to the workspace for the combine kernel.

struct CtaPlan {
  int64_t U;
  int64_t ps_first;  // first page of sequence b_first in the concatenation
  int32_t R;
  int32_t b_first;
};

// Pages of sequence b: 0 for a non-positive length, at most max_pages.
IRIS_DEV int32_t seq_pages(const DecodeParams& p, int b) {
  const int32_t L = p.seq_lens[b];
  if (L <= 0) return 0;
  const int32_t np = (L + kPage - 1) / kPage;
  return np < p.max_pages ? np : p.max_pages;
}

// Batches of at most 32 * kPlanPerLane sequences: lane l takes sequences
// [l*K, l*K + K), K = ceil(batch / 32), loads all their lengths at once (one
// memory round trip instead of two dependent passes) and keeps the page
// counts in registers for the prefix scan and for finding the range's first
// sequence.
constexpr int kPlanPerLane = 8;

IRIS_DEV void plan_cta_regs(const DecodeParams& p, int r, int ranges, bool leader, int lane, CtaPlan* out) {
  const int K = (p.batch + 31) / 32;
  const int b0 = lane * K;
  int32_t np[kPlanPerLane];
#pragma unroll
  for (int j = 0; j < kPlanPerLane; ++j) {
    const int b = b0 + j;
    np[j] = (j < K && b < p.batch) ? __ldg(p.seq_lens + b) : 0;
  }
  int32_t tot = 0;
#pragma unroll
  for (int j = 0; j < kPlanPerLane; ++j) {
    const int b = b0 + j;
    const int32_t L = np[j];
    int32_t n = 0;
    if (j < K && b < p.batch) {
      if (L <= 0) {
        if (leader) set_error(p.err, IRIS_ERR_SEQ_LEN);
      } else {
        n = (L + kPage - 1) / kPage;
        if (n > p.max_pages) {
          if (leader) set_error(p.err, IRIS_ERR_BLOCK_TABLE);
          n = p.max_pages;
        }
      }
    }
    np[j] = n;
    tot += n;
  }
  int32_t x = tot;  // inclusive scan of the lanes' totals
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  const int32_t excl = x - tot;
  const int64_t U = __shfl_sync(0xffffffffu, x, 31);
  if (leader) {
    int32_t run = excl;
#pragma unroll
    for (int j = 0; j < kPlanPerLane; ++j) {
      if (j < K && b0 + j < p.batch) const_cast<int32_t*>(p.prefix)[b0 + j] = run;
      run += np[j];
    }
  }
  int32_t R = 0;
  if (U > 0) {
    const int64_t want = wanted_ranges(U);
    R = static_cast<int32_t>(want < ranges ? want : ranges);
  }
  if (leader && lane == 0) {
    const_cast<int32_t*>(p.prefix)[p.batch] = static_cast<int32_t>(U);
    const_cast<int32_t*>(p.meta)[0] = static_cast<int32_t>(U);
    const_cast<int32_t*>(p.meta)[1] = R;
  }
  int32_t bf = 0, psf = 0;
  if (r < R) {
    // the sequence holding page u0: the first b whose pages end past u0
    const int64_t u0 = range_start(r, U, R);
    const unsigned hit = __ballot_sync(0xffffffffu, static_cast<int64_t>(x) > u0);
    const int i = __ffs(hit) - 1;
    int32_t run = excl, mb = 0, mps = 0;
    bool found = false;
#pragma unroll
    for (int j = 0; j < kPlanPerLane; ++j) {
      if (!found && static_cast<int64_t>(run) + np[j] > u0) {
        found = true;
        mb = b0 + j;
        mps = run;
      }
      run += np[j];
    }
    bf = __shfl_sync(0xffffffffu, mb, i);
    psf = __shfl_sync(0xffffffffu, mps, i);
  }
  if (lane == 0) {
    out->U = U;
    out->R = R;
    out->b_first = bf;
    out->ps_first = psf;
  }
}

IRIS_DEV void plan_cta(const DecodeParams& p, int r, int ranges, bool leader, int lane, CtaPlan* out) {
  if (p.batch <= 32 * kPlanPerLane) {
    plan_cta_regs(p, r, ranges, leader, lane, out);
    return;
  }
  int64_t U = 0;
  for (int base = 0; base < p.batch; base += 32) {
    const int b = base + lane;
    int32_t np = 0;
    if (b < p.batch) {
      const int32_t L = p.seq_lens[b];
      if (L <= 0) {
        if (leader) set_error(p.err, IRIS_ERR_SEQ_LEN);
      } else {
        np = (L + kPage - 1) / kPage;
        if (np > p.max_pages) {
          if (leader) set_error(p.err, IRIS_ERR_BLOCK_TABLE);
          np = p.max_pages;
        }
      }
    }
    int32_t x = np;  // inclusive warp scan
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int32_t y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (leader && b < p.batch) const_cast<int32_t*>(p.prefix)[b] = static_cast<int32_t>(U + x - np);
    U += __shfl_sync(0xffffffffu, x, 31);
  }
  int32_t R = 0;
  if (U > 0) {
    const int64_t want = wanted_ranges(U);
    R = static_cast<int32_t>(want < ranges ? want : ranges);
  }
  if (leader && lane == 0) {
    const_cast<int32_t*>(p.prefix)[p.batch] = static_cast<int32_t>(U);
    const_cast<int32_t*>(p.meta)[0] = static_cast<int32_t>(U);
    const_cast<int32_t*>(p.meta)[1] = R;
  }
  int32_t bf = 0;
  int64_t psf = 0;
  if (r < R) {
    // the sequence holding page u0: the first b whose pages end past u0
    const int64_t u0 = range_start(r, U, R);
    int64_t carry = 0;
    for (int base = 0; base < p.batch; base += 32) {
      const int b = base + lane;
      const int32_t np = b < p.batch ? seq_pages(p, b) : 0;
      int32_t x = np;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int32_t y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
      }
      const unsigned hit = __ballot_sync(0xffffffffu, b < p.batch && carry + x > u0);
      if (hit) {
        const int i = __ffs(hit) - 1;
        bf = base + i;
        psf = carry + __shfl_sync(0xffffffffu, x - np, i);
        break;
      }
      carry += __shfl_sync(0xffffffffu, x, 31);
    }
  }
  if (lane == 0) {
    out->U = U;
    out->R = R;
    out->b_first = bf;
    out->ps_first = psf;
  }
}

// Per-warp attention state for one (sequence piece, KV head).
template <int D, int NT>
struct WarpState {
  float o[NT][D / 16][4];
  float m[NT][2];
  float l[NT][2];
  uint32_t qf[NT][D / 16][2];       // Q as mma B fragments (permuted dims, odd dims / 16)
  float corr[NT][D / 32][2];        // bias correction per (group, column)
};

// Load query heads [h0, h0+qpk) of sequence b as B fragments and derive the
// per-group bias corrections.  Lane (n = lane/4, t = lane%4) owns query head
// n of each n-tile and dims 8t..8t+7 of every 32-dim group.
template <int D, int NT>
IRIS_DEV void load_query(WarpState<D, NT>& st, const __half* __restrict__ q_seq, int qpk, int lane) {
  const int n = lane >> 2, t = lane & 3;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int qh = nt * 8 + n;
#pragma unroll
    for (int g = 0; g < D / 32; ++g) {
      uint4 raw = make_uint4(0, 0, 0, 0);
      if (qh < qpk) raw = *reinterpret_cast<const uint4*>(q_seq + qh * D + g * 32 + t * 8);
      const __half* e = reinterpret_cast<const __half*>(&raw);
      const __half s16 = __float2half_rn(0.0625f);
      __half eo[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) eo[i] = __hmul(e[2 * i + 1], s16);  // odd dims / 16 (exact)
      st.qf[nt][2 * g + 0][0] = h2_as_u32(__halves2half2(e[0], e[4]));
      st.qf[nt][2 * g + 0][1] = h2_as_u32(__halves2half2(eo[0], eo[2]));
      st.qf[nt][2 * g + 1][0] = h2_as_u32(__halves2half2(e[2], e[6]));
      st.qf[nt][2 * g + 1][1] = h2_as_u32(__halves2half2(eo[1], eo[3]));
      float c = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        c += 1032.0f * __half2float(e[2 * i]);
        c += 1152.0f * __half2float(eo[i]);
      }
      c += __shfl_xor_sync(0xffffffffu, c, 1);
      c += __shfl_xor_sync(0xffffffffu, c, 2);
      // column j of this lane's C fragment is query head 2t + j
      st.corr[nt][g][0] = __shfl_sync(0xffffffffu, c, (2 * t) * 4);
      st.corr[nt][g][1] = __shfl_sync(0xffffffffu, c, (2 * t + 1) * 4);
    }
#pragma unroll
    for (int i = 0; i < D / 16; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) st.o[nt][i][j] = 0.f;
    st.m[nt][0] = st.m[nt][1] = kNegInf;
    st.l[nt][0] = st.l[nt][1] = 0.f;
  }
}

// Shared-memory layout of a stage's K (or V) tiles for the CTA's block of
// HB KV heads, and each lane's ldmatrix.x4 address in it.  The four 8x8
// matrices of one ldmatrix.x4 cover token rows 8*((l>>3)&1).. and 16-byte
// segments 2*i + (l>>4) of head g's D/2-byte row.
//  * R128 = false: one [16 tokens][D/2 bytes] tile per head, swizzled by the
//    tensor map's 64-byte (D = 128) or 32-byte (D = 64) pattern.
//  * R128 = true: one [16 tokens][128 bytes] tile per kRowHeads = 256 / D
//    adjacent heads (a 128-byte row holds one token of all of them, as the
//    cache stores it), swizzled by the 128-byte pattern: 16-byte chunk c of
//    row r sits at chunk c ^ (r & 7).  Whole 128-byte rows make the TMA's
//    transactions whole lines.
// lane_off(lane, g) is the offset of segment pair 0 of head g; the segment-
// pair bit is disjoint from the others, so pair i is at lane_off ^ (32 * i)
// (also after adding a 1-KB aligned stage base).
template <int D, bool R128>
struct KvTiles {
  static constexpr int kTile = kPage * D / 2;  // bytes of one head per page
  static constexpr int kRowHeads = 256 / D;    // heads per 128-byte row (R128)
  IRIS_DEV static uint32_t lane_off(int lane, int g) {
    const int mat = lane >> 3;
    const int row = (lane & 7) + 8 * (mat & 1);
    if constexpr (R128) {
      const uint32_t unit = static_cast<uint32_t>(g / kRowHeads) * (kRowHeads * kTile);
      const int chunk = (g % kRowHeads) * (D / 32) + (mat >> 1);
      return unit + row * 128 + ((chunk ^ (lane & 7)) << 4);
    } else {
      const int sw = D == 128 ? ((row >> 1) & 3) : ((row >> 2) & 1);  // TMA SWIZZLE_64B / SWIZZLE_32B
      return static_cast<uint32_t>(g) * kTile + row * (D / 2) + (((mat >> 1) ^ sw) << 4);
    }
  }
};

// One page (16 tokens) of one KV head.
// Scores of one page (16 tokens) for this warp's KV head:
// s[nt][0..3] = S^T[token g8 / g8+8][query head 2t / 2t+1] (unscaled logits).
// ktile / ksc are shared-memory addresses of the head's K tile and of its
// column in the page's K scale block (row stride `scale_stride` bytes).
template <int D, int NT>
IRIS_DEV void page_scores(const WarpState<D, NT>& st, uint32_t ktile, uint32_t ksc, int scale_stride, int lane,
                          float (&s)[NT][4]) {
  constexpr int G = D / 32;
  const int g8 = lane >> 2;
  // kw[grp][0] = token g8, kw[grp][1] = token g8 + 8 (32 dims of group grp)
  uint32_t kw[G][2];
#pragma unroll
  for (int i = 0; i < G / 2; ++i) {
    uint32_t r[4];
    ldmatrix_x4(r, ktile ^ (32u * i));
    kw[2 * i][0] = r[0];
    kw[2 * i][1] = r[1];
    kw[2 * i + 1][0] = r[2];
    kw[2 * i + 1][1] = r[3];
  }
  float ks[2][G];
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    const uint32_t sp = ksc + (g8 + 8 * rr) * scale_stride;
    if constexpr (G == 4) {
      const uint2 u = lds64(sp);
      const float2 a = __half22float2(u32_as_h2(u.x)), b = __half22float2(u32_as_h2(u.y));
      ks[rr][0] = a.x; ks[rr][1] = a.y; ks[rr][2] = b.x; ks[rr][3] = b.y;
    } else {
      const float2 a = __half22float2(u32_as_h2(lds32(sp)));
      ks[rr][0] = a.x; ks[rr][1] = a.y;
    }
  }
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float acc[4] = {-st.corr[nt][g][0], -st.corr[nt][g][1], -st.corr[nt][g][0], -st.corr[nt][g][1]};
#pragma unroll
      for (int sub = 0; sub < 2; ++sub) {
        const uint32_t w0 = kw[g][0] >> (8 * sub), w1 = kw[g][1] >> (8 * sub);
        const uint32_t a[4] = {int4_lo_biased(w0), int4_lo_biased(w1), int4_hi_biased(w0), int4_hi_biased(w1)};
        mma_16816(acc, a, st.qf[nt][2 * g + sub][0], st.qf[nt][2 * g + sub][1], acc);
      }
      if (g == 0) {
        s[nt][0] = ks[0][g] * acc[0];
        s[nt][1] = ks[0][g] * acc[1];
        s[nt][2] = ks[1][g] * acc[2];
        s[nt][3] = ks[1][g] * acc[3];
      } else {
        s[nt][0] = fmaf(ks[0][g], acc[0], s[nt][0]);
        s[nt][1] = fmaf(ks[0][g], acc[1], s[nt][1]);
        s[nt][2] = fmaf(ks[1][g], acc[2], s[nt][2]);
        s[nt][3] = fmaf(ks[1][g], acc[3], s[nt][3]);
      }
    }
  }
}

// O += V^T P'^T for one page.  p[nt][0..3] are this lane's probabilities in
// the score layout; tokens >= `valid` get a zero V scale when MASK (their
// slots may hold garbage, even NaN scales).
template <int D, int NT, bool MASK>
IRIS_DEV void page_pv(WarpState<D, NT>& st, uint32_t vtile, uint32_t vsc, int scale_stride, int valid,
                      const float (&p)[NT][4], int lane) {
  constexpr int G = D / 32;
  const int t = lane & 3;
  // V scales of tokens 2t, 2t+1, 2t+8, 2t+9 as half2 (token a, token b) per group
  uint32_t sv01[G], sv89[G];
  {
    uint32_t raw[4][G / 2];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int tok = 2 * t + (k & 1) + 8 * (k >> 1);
      const uint32_t sp = vsc + tok * scale_stride;
      const bool ok = !MASK || tok < valid;
      if constexpr (G == 4) {
        const uint2 u = lds64(sp);
        raw[k][0] = ok ? u.x : 0u;
        raw[k][1] = ok ? u.y : 0u;
      } else {
        const uint32_t u = lds32(sp);
        raw[k][0] = ok ? u : 0u;
      }
    }
#pragma unroll
    for (int j = 0; j < G / 2; ++j) {
      sv01[2 * j] = prmt(raw[0][j], raw[1][j], 0x5410);
      sv01[2 * j + 1] = prmt(raw[0][j], raw[1][j], 0x7632);
      sv89[2 * j] = prmt(raw[2][j], raw[3][j], 0x5410);
      sv89[2 * j + 1] = prmt(raw[2][j], raw[3][j], 0x7632);
    }
  }
  // P^T as B operands via an in-register 8x8 transpose
  uint32_t pb[NT][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    pb[nt][0] = movmatrix_trans(h2_as_u32(__floats2half2_rn(p[nt][0], p[nt][1])));
    pb[nt][1] = movmatrix_trans(h2_as_u32(__floats2half2_rn(p[nt][2], p[nt][3])));
  }
#pragma unroll
  for (int i = 0; i < G / 2; ++i) {
    uint32_t r[4];
    ldmatrix_x4_trans(r, vtile ^ (32u * i));
    // r[0] = (tokens 2t,2t+1; group 2i), r[1] = (tokens 2t+8,2t+9; group 2i),
    // r[2], r[3] likewise for group 2i+1
#pragma unroll
    for (int gg = 0; gg < 2; ++gg) {
      const int g = 2 * i + gg;
      const uint32_t wa = r[2 * gg], wb = r[2 * gg + 1];
      uint32_t bv[NT][2];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        bv[nt][0] = h2_as_u32(__hmul2(u32_as_h2(pb[nt][0]), u32_as_h2(sv01[g])));
        bv[nt][1] = h2_as_u32(__hmul2(u32_as_h2(pb[nt][1]), u32_as_h2(sv89[g])));
      }
#pragma unroll
      for (int jj = 0; jj < 2; ++jj) {
        const uint32_t xa = wa >> (8 * jj), xb = wb >> (8 * jj);
        const uint32_t a[4] = {int4_lo_exact(xa), int4_hi_exact(xa), int4_lo_exact(xb), int4_hi_exact(xb)};
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) mma_16816(st.o[nt][2 * g + jj], a, bv[nt][0], bv[nt][1], st.o[nt][2 * g + jj]);
      }
    }
  }
}

// NPG consecutive pages (1 or 2) of this warp's KV head with one online-
// softmax update.  base[i] is the shared address of page i's stage; `valid`
// counts the sequence's tokens from page 0 on (MASK: fewer than 16*NPG).
template <int D, int NT, int NPG, bool MASK>
IRIS_DEV void process_pages(WarpState<D, NT>& st, const uint32_t (&base)[NPG], uint32_t k_off, uint32_t v_off,
                            uint32_t ks_off, uint32_t vs_off, int scale_stride, int valid, float scale_log2,
                            int lane) {
  const int g8 = lane >> 2;
  float x[NPG][NT][4];
#pragma unroll
  for (int pi = 0; pi < NPG; ++pi) {
    page_scores<D, NT>(st, base[pi] + k_off, base[pi] + ks_off, scale_stride, lane, x[pi]);
    const bool r0 = !MASK || g8 + 16 * pi < valid, r1 = !MASK || g8 + 8 + 16 * pi < valid;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      x[pi][nt][0] = r0 ? x[pi][nt][0] * scale_log2 : kNegInf;
      x[pi][nt][1] = r0 ? x[pi][nt][1] * scale_log2 : kNegInf;
      x[pi][nt][2] = r1 ? x[pi][nt][2] * scale_log2 : kNegInf;
      x[pi][nt][3] = r1 ? x[pi][nt][3] * scale_log2 : kNegInf;
    }
  }
  float p[NPG][NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    float mx0 = fmaxf(x[0][nt][0], x[0][nt][2]), mx1 = fmaxf(x[0][nt][1], x[0][nt][3]);
#pragma unroll
    for (int pi = 1; pi < NPG; ++pi) {
      mx0 = fmaxf(mx0, fmaxf(x[pi][nt][0], x[pi][nt][2]));
      mx1 = fmaxf(mx1, fmaxf(x[pi][nt][1], x[pi][nt][3]));
    }
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
    }
    const float mn0 = fmaxf(st.m[nt][0], mx0), mn1 = fmaxf(st.m[nt][1], mx1);
    if (__any_sync(0xffffffffu, (mn0 > st.m[nt][0]) || (mn1 > st.m[nt][1]))) {
      const float c0 = ex2(st.m[nt][0] - mn0), c1 = ex2(st.m[nt][1] - mn1);  // ex2(-inf) = 0
#pragma unroll
      for (int i = 0; i < D / 16; ++i) {
        st.o[nt][i][0] *= c0;
        st.o[nt][i][1] *= c1;
        st.o[nt][i][2] *= c0;
        st.o[nt][i][3] *= c1;
      }
      st.l[nt][0] *= c0;
      st.l[nt][1] *= c1;
      st.m[nt][0] = mn0;
      st.m[nt][1] = mn1;
    }
#pragma unroll
    for (int pi = 0; pi < NPG; ++pi) {
      p[pi][nt][0] = ex2(x[pi][nt][0] - st.m[nt][0]);
      p[pi][nt][1] = ex2(x[pi][nt][1] - st.m[nt][1]);
      p[pi][nt][2] = ex2(x[pi][nt][2] - st.m[nt][0]);
      p[pi][nt][3] = ex2(x[pi][nt][3] - st.m[nt][1]);
      st.l[nt][0] += p[pi][nt][0] + p[pi][nt][2];
      st.l[nt][1] += p[pi][nt][1] + p[pi][nt][3];
    }
  }
#pragma unroll
  for (int pi = 0; pi < NPG; ++pi)
    page_pv<D, NT, MASK>(st, base[pi] + v_off, base[pi] + vs_off, scale_stride, valid - 16 * pi, p[pi], lane);
}

// Finish a (sequence piece, KV head): reduce l over the lane's token rows,
// then either write the final output or a partial record.
template <int D, int NT>
IRIS_DEV void finish_piece(const DecodeParams& p, WarpState<D, NT>& st, int b, int kvh, bool complete, int64_t rec,
                           int lane) {
  const int g8 = lane >> 2, t = lane & 3;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    float l0 = st.l[nt][0], l1 = st.l[nt][1];
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      l0 += __shfl_xor_sync(0xffffffffu, l0, o);
      l1 += __shfl_xor_sync(0xffffffffu, l1, o);
    }
    const float inv[2] = {1.0f / l0, 1.0f / l1};
    const float lse[2] = {st.m[nt][0] + lg2(l0), st.m[nt][1] + lg2(l1)};
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int qh_local = nt * 8 + 2 * t + j;
      if (qh_local >= p.qpk) continue;
      const int qh = kvh * p.qpk + qh_local;
#pragma unroll
      for (int g = 0; g < D / 32; ++g) {
        // dims 32g + 4*g8 + {0,1,2,3} from m-tiles (2g, 2g+1), rows (g8, g8+8)
        const float v0 = st.o[nt][2 * g][j] * inv[j];
        const float v1 = st.o[nt][2 * g][2 + j] * inv[j];
        const float v2 = st.o[nt][2 * g + 1][j] * inv[j];
        const float v3 = st.o[nt][2 * g + 1][2 + j] * inv[j];
        const int d = 32 * g + 4 * g8;
        if (complete && p.out_mode == IRIS_DECODE_OUT_FP16) {
          __half* dst = static_cast<__half*>(p.out) + (static_cast<int64_t>(b) * p.hq + qh) * D + d;
          uint2 u;
          u.x = h2_as_u32(__floats2half2_rn(v0, v1));
          u.y = h2_as_u32(__floats2half2_rn(v2, v3));
          *reinterpret_cast<uint2*>(dst) = u;
        } else {
          float* dst = complete ? static_cast<float*>(p.out) + (static_cast<int64_t>(b) * p.hq + qh) * D + d
                                : p.rec_o + (rec * p.hq + qh) * D + d;
          *reinterpret_cast<float4*>(dst) = make_float4(v0, v1, v2, v3);
        }
      }
      if (g8 == 0) {
        if (complete) {
          if (p.out_mode == IRIS_DECODE_OUT_LSE) p.out_lse[static_cast<int64_t>(b) * p.hq + qh] = lse[j];
        } else {
          p.rec_lse[rec * p.hq + qh] = lse[j];
        }
      }
    }
  }
}

// The producer warp of a decode CTA: walks the CTA's page range, fetches
// and validates page ids 32 at a time (all lanes, one chunk ahead), and lane 0
// waits for free ring stages and issues, per page, one 4-D TMA copy per
// tensor for the CTA's HB heads plus the page's two scale blocks.  Returns
// once every copy it issued has landed (or a bounded wait gave up).
// How a stage's tiles are fetched: the INT4 cache (4-D box per tensor plus
// the page's two scale blocks) or the FP16 cache (4-D box at D = 64, 5-D box
// of two 128-byte halves per row at D = 128; no scales).
// kRowHeads: heads per box row (1: one head's D/2 bytes per row; 256 / D:
// 128-byte rows of kRowHeads heads), so the box's third coordinate is the
// first head / kRowHeads.
template <int kRowHeads>
struct Int4Copy {
  static constexpr bool kScales = true;
  IRIS_DEV static void load(void* dst, const CUtensorMap* m, int head0, int pid, uint64_t* bar) {
    tma_load_4d(dst, m, 0, 0, head0 / kRowHeads, pid, bar);
  }
};
template <int kDims>
struct Fp16Copy {
  static constexpr bool kScales = false;
  IRIS_DEV static void load(void* dst, const CUtensorMap* m, int head0, int pid, uint64_t* bar) {
    if constexpr (kDims == 5)
      tma_load_5d(dst, m, 0, 0, 0, head0, pid, bar);
    else
      tma_load_4d(dst, m, 0, 0, head0, pid, bar);
  }
};

template <typename Copy, int kTile>
IRIS_DEV void run_producer(const CUtensorMap* kmap_p, const CUtensorMap* vmap_p, const DecodeParams& p,
                           uint8_t* smem, int stage_bytes, int S, int HB, int hblk, int64_t u0, int64_t u1,
                           int b_first, int64_t ps_first, uint64_t* full, uint32_t full_u32, uint32_t empty_u32,
                           int scale_block, int lane) {
  // All lanes fetch (and validate) page ids 32 at a time, one chunk ahead
  // of lane 0, which waits for free stages and issues the copies.
  if (lane == 0) {
    prefetch_tensormap(kmap_p);
    prefetch_tensormap(vmap_p);
  }
  const uint32_t tx = 2 * HB * kTile + (Copy::kScales ? 2 * scale_block : 0);
  uint32_t issued = 0;
  int s = 0;          // stage of the next page
  uint32_t ph = 0;    // its ring pass parity
  bool alive = true;
  int b = b_first;
  int64_t ps = ps_first;  // first page of sequence b
  int64_t u = u0;
  auto fetch_ids = [&](const int32_t* row, int64_t first, int64_t count) -> int32_t {
    int32_t pid = 0;
    if (lane < count) {
      pid = row[first + lane];
      if (pid < 0 || static_cast<int64_t>(pid) >= p.num_pages) {
        set_error(p.err, IRIS_ERR_PAGE_ID);
        pid = 0;  // stay in bounds; the error word makes the call fail
      }
    }
    return pid;
  };
  while (alive && u < u1) {
    const int64_t pe = ps + seq_pages(p, b);
    if (pe <= u) {
      ps = pe;
      ++b;
      continue;
    }
    const int64_t hi = pe < u1 ? pe : u1;
    const int32_t* bt_row = p.block_table + static_cast<int64_t>(b) * p.bt_stride;
    int64_t chunk = u;
    int32_t ids = fetch_ids(bt_row, chunk - ps, hi - chunk);
    while (chunk < hi) {
      const int n = static_cast<int>(hi - chunk < 32 ? hi - chunk : 32);
      const int64_t next = chunk + n;
      const int32_t ids_next = next < hi ? fetch_ids(bt_row, next - ps, hi - next) : 0;
      for (int j = 0; j < n; ++j) {
        const int32_t pid = __shfl_sync(0xffffffffu, ids, j);
        if (lane == 0 && alive) {
          if (!mbar_wait_bounded(empty_u32 + 8 * s, ph ^ 1, p.err)) {
            alive = false;
          } else {
            uint8_t* st = smem + s * stage_bytes;
            mbar_arrive_expect_tx(full + s, tx);
            Copy::load(st, kmap_p, hblk * HB, pid, full + s);
            Copy::load(st + HB * kTile, vmap_p, hblk * HB, pid, full + s);
            if constexpr (Copy::kScales) {
              uint8_t* sc = st + 2 * HB * kTile;
              bulk_g2s(sc, p.k_scale + static_cast<int64_t>(pid) * scale_block, scale_block, full + s);
              bulk_g2s(sc + scale_block, p.v_scale + static_cast<int64_t>(pid) * scale_block, scale_block,
                       full + s);
            }
            ++issued;
          }
        }
        if (++s == S) { s = 0; ph ^= 1; }
      }
      alive = __shfl_sync(0xffffffffu, alive, 0);
      if (!alive) break;
      ids = ids_next;
      chunk = next;
    }
    u = hi;
    ps = pe;
    ++b;
  }
  // drain: every copy this CTA issued has landed before it exits
  if (lane == 0) {
    const uint32_t last = issued;  // stages are issued in order, so the last S are [issued - S, issued)
    const uint32_t first = last > static_cast<uint32_t>(S) ? last - S : 0;
    for (uint32_t k = first; k < last; ++k) mbar_wait_bounded(full_u32 + 8 * (k % S), (k / S) & 1, p.err);
  }
}

template <int D, int NT, bool R128>
__global__ void __maxnreg__(128) decode_kernel(const __grid_constant__ CUtensorMap kmap,
                                                        const __grid_constant__ CUtensorMap vmap,
                                                        const DecodeParams p) {
  using C = DecCfg<D>;
  grid_dependents_launch();  // the combine kernel may launch and wait meanwhile
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

  const int hblk = blockIdx.x;
  const int r = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int HB = p.hb;
  const int S = p.stages;
  __shared__ CtaPlan plan;

  const int scale_block = kPage * p.hkv * C::kGroups * 2;  // bytes of one page's K (or V) scales
  const int stage_bytes = ((2 * HB * C::kTileBytes + 2 * scale_block) + 1023) & ~1023;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * stage_bytes);
  uint64_t* empty = full + S;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, HB);
    }
    fence_barrier_init();
  }
  if (warp == 0) plan_cta(p, r, gridDim.y, blockIdx.x == 0 && r == 0, lane, &plan);
  __syncthreads();
  const int64_t U = plan.U;
  const int R = plan.R;
  if (r >= R) return;  // uniform per CTA (nothing was issued yet)

  const int64_t u0 = range_start(r, U, R), u1 = range_start(r + 1, U, R);
  const int b_first = plan.b_first;
  const int64_t ps_first = plan.ps_first;
  const uint32_t full_u32 = smem_u32(full), empty_u32 = smem_u32(empty);

  if (warp == HB) {
    run_producer<Int4Copy<R128 ? 256 / D : 1>, C::kTileBytes>(&kmap, &vmap, p, smem, stage_bytes, S, HB, hblk, u0,
                                                              u1, b_first, ps_first, full, full_u32, empty_u32,
                                                              scale_block, lane);
    return;
  }

  // ========================= consumer warps =========================
  const int kvh = hblk * HB + warp;
  WarpState<D, NT> st;
  const uint32_t ring = smem_u32(smem);
  // this warp's tiles and scale columns, relative to a stage's base
  // this lane's ldmatrix addresses of the warp's head, relative to a stage's base
  const uint32_t k_off = KvTiles<D, R128>::lane_off(lane, warp), v_off = HB * C::kTileBytes + k_off;
  const uint32_t ks_off = 2 * HB * C::kTileBytes + kvh * C::kGroups * 2;
  const uint32_t vs_off = ks_off + scale_block;
  const int scale_stride = p.hkv * C::kGroups * 2;
  int s = 0;
  uint32_t ph = 0;
  uint32_t stage = ring;  // base address of stage s
  int b = b_first;
  int64_t ps = ps_first;  // first page of sequence b
  int64_t u = u0;
  while (u < u1) {
    const int64_t pe = ps + seq_pages(p, b);
    if (pe <= u) {
      ps = pe;
      ++b;
      continue;
    }
    const int64_t hi = pe < u1 ? pe : u1;
    const int L = min(p.seq_lens[b], p.max_pages * kPage);
    load_query<D, NT>(st, p.query + (static_cast<int64_t>(b) * p.hq + kvh * p.qpk) * D, p.qpk, lane);
    int valid = L - static_cast<int>(u - ps) * kPage;  // tokens left from this page on
    int left = static_cast<int>(hi - u);                 // pages of this piece still to do
    while (left > 0) {
      // two pages per softmax update where the registers allow it (NT == 1)
      if (NT == 1 && left >= 2) {
        const int s1 = s + 1 == S ? 0 : s + 1;
        const uint32_t ph1 = s + 1 == S ? ph ^ 1 : ph;
        const uint32_t base[2] = {stage, s1 == 0 ? ring : stage + stage_bytes};
        if (!mbar_wait_bounded(full_u32 + 8 * s, ph, p.err)) return;
        if (!mbar_wait_bounded(full_u32 + 8 * s1, ph1, p.err)) return;
        if (valid >= 2 * kPage)
          process_pages<D, NT, 2, false>(st, base, k_off, v_off, ks_off, vs_off, scale_stride, valid, p.scale_log2,
                                         lane);
        else
          process_pages<D, NT, 2, true>(st, base, k_off, v_off, ks_off, vs_off, scale_stride, valid, p.scale_log2,
                                        lane);
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(empty_u32 + 8 * s);
          mbar_arrive(empty_u32 + 8 * s1);
        }
        valid -= 2 * kPage;
        left -= 2;
        if (s1 + 1 == S) {
          s = 0;
          stage = ring;
        } else {
          s = s1 + 1;
          stage = base[1] + stage_bytes;
        }
        ph = (s1 + 1 == S) ? ph1 ^ 1 : ph1;
      } else {
        const uint32_t base[1] = {stage};
        if (!mbar_wait_bounded(full_u32 + 8 * s, ph, p.err)) return;
        if (valid >= kPage)
          process_pages<D, NT, 1, false>(st, base, k_off, v_off, ks_off, vs_off, scale_stride, valid, p.scale_log2,
                                         lane);
        else
          process_pages<D, NT, 1, true>(st, base, k_off, v_off, ks_off, vs_off, scale_stride, valid, p.scale_log2,
                                        lane);
        __syncwarp();
        if (lane == 0) mbar_arrive(empty_u32 + 8 * s);
        valid -= kPage;
        left -= 1;
        if (++s == S) {
          s = 0;
          ph ^= 1;
          stage = ring;
        } else {
          stage += stage_bytes;
        }
      }
    }
    const bool complete = (ps >= u0) && (pe <= u1);
    const int64_t rec = static_cast<int64_t>(r) * 2 + (u == u0 ? 0 : 1);
    finish_piece<D, NT>(p, st, b, kvh, complete, rec, lane);
    u = hi;
    ps = pe;
    ++b;
  }
}

// ------------------------------------------------- head-pair consumer path
// For GQA groups of at most 4 query heads the MMA's 8 columns would be half
// empty with one KV head per warp.  Here a warp owns HP = 8 / CW KV heads
// and column c of every fragment belongs to KV head c / CW (query head
// c % CW of it; CW = 4 or 2 columns per head, columns past the group size are
// zero).  Scores: one accumulator per 32-dim group collects, head by head,
// K_h . Q_h^T where head h's B operand is the query tile with every other
// head's columns read as zeros, so each column receives only its own head's
// products.  PV: O^T += V_h^T . P'_h^T with P' zeroed outside head h's
// columns.  Softmax state, scale products and the rescaling of O are shared
// by the HP heads, and O takes 32 registers for all of them.
//
// The query tile lives in shared memory (8 rows = columns x D halves, in the
// k order of the QK MMAs, 16-byte chunks XOR-swizzled by row) and is read
// with ldmatrix; lanes whose row belongs to another head point at a 256-byte
// zero block instead.

template <int D>
struct PairState {
  float o[D / 16][4];
  float m[2];
  float l[2];
  float ncorr[D / 32][2];  // minus the bias correction per (group, column)
};

// Write the warp's query tile (heads kv0 .. kv0+HP-1 of sequence b) and
// derive the bias corrections.  Lane (n = lane/4, t = lane%4) handles row n
// and dims 8t..8t+7 of every 32-dim group.
template <int D, int HP>
IRIS_DEV void pair_load_query(PairState<D>& st, const __half* __restrict__ q_seq, int kv0, int qpk, uint32_t qtile,
                              int lane) {
  constexpr int CW = 8 / HP;
  const int n = lane >> 2, t = lane & 3;
  const int qi = n % CW;
  const __half* qrow = q_seq + ((kv0 + n / CW) * qpk + qi) * D;
  const uint32_t row = qtile + n * (2 * D);
#pragma unroll
  for (int g = 0; g < D / 32; ++g) {
    uint4 raw = make_uint4(0, 0, 0, 0);
    if (qi < qpk) raw = *reinterpret_cast<const uint4*>(qrow + g * 32 + t * 8);
    const __half* e = reinterpret_cast<const __half*>(&raw);
    const __half s16 = __float2half_rn(0.0625f);
    __half eo[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) eo[i] = __hmul(e[2 * i + 1], s16);  // odd dims / 16 (exact)
    // k-step 2g+sub: k = 2t, 2t+1 <- even dims 8t+2sub, 8t+2sub+4 (chunk 2ks);
    //                k = 8+2t, 9+2t <- odd dims / 16 (chunk 2ks+1)
#pragma unroll
    for (int sub = 0; sub < 2; ++sub) {
      const int ks = 2 * g + sub;
      const uint32_t w0 = h2_as_u32(__halves2half2(e[2 * sub], e[2 * sub + 4]));
      const uint32_t w1 = h2_as_u32(__halves2half2(eo[sub], eo[sub + 2]));
      sts32(row + (((2 * ks) ^ n) << 4) + 4 * t, w0);
      sts32(row + (((2 * ks + 1) ^ n) << 4) + 4 * t, w1);
    }
    float c = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      c += 1032.0f * __half2float(e[2 * i]);
      c += 1152.0f * __half2float(eo[i]);
    }
    c += __shfl_xor_sync(0xffffffffu, c, 1);
    c += __shfl_xor_sync(0xffffffffu, c, 2);
    // column j of this lane's C fragment is row 2t + j of the tile
    st.ncorr[g][0] = -__shfl_sync(0xffffffffu, c, (2 * t) * 4);
    st.ncorr[g][1] = -__shfl_sync(0xffffffffu, c, (2 * t + 1) * 4);
  }
#pragma unroll
  for (int i = 0; i < D / 16; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) st.o[i][j] = 0.f;
  st.m[0] = st.m[1] = 0.f;  // replaced by the first page's maxima
  st.l[0] = st.l[1] = 0.f;
  __syncwarp();
}

// Scores of one page for the warp's HP heads: s[0..3] = S^T[token g8 / g8+8]
// [column 2t / 2t+1] (unscaled logits).  ktile0: shared address of the first
// head's K tile (heads follow at kTileBytes); qaddr[h]: this lane's ldmatrix
// row address for head h's (masked) query tile, XOR 64*i selecting k-steps
// 2i, 2i+1; ksc: the lane's head's column in the page's K scale block.
template <int D, int HP>
IRIS_DEV void pair_page_scores(const PairState<D>& st, uint32_t stage, const uint32_t (&klane)[HP],
                               const uint32_t (&qaddr)[HP], uint32_t ksc, int scale_stride, int lane, float (&s)[4]) {
  constexpr int G = D / 32;
  const int g8 = lane >> 2;
  float ks[2][G];
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    const uint32_t sp = ksc + (g8 + 8 * rr) * scale_stride;
    if constexpr (G == 4) {
      const uint2 u = lds64(sp);
      const float2 a = __half22float2(u32_as_h2(u.x)), b = __half22float2(u32_as_h2(u.y));
      ks[rr][0] = a.x; ks[rr][1] = a.y; ks[rr][2] = b.x; ks[rr][3] = b.y;
    } else {
      const float2 a = __half22float2(u32_as_h2(lds32(sp)));
      ks[rr][0] = a.x; ks[rr][1] = a.y;
    }
  }
#pragma unroll
  for (int i = 0; i < G / 2; ++i) {
    // groups 2i, 2i+1 of every head; the first MMA of a group reads its
    // seed (minus the bias correction) straight from the state
    float acc[2][4];
#pragma unroll
    for (int h = 0; h < HP; ++h) {
      uint32_t kr[4];
      ldmatrix_x4(kr, (stage + klane[h]) ^ (32u * i));
#pragma unroll
      for (int gg = 0; gg < 2; ++gg) {
        uint32_t qb[4];  // (b0, b1) of k-steps 2g, 2g+1 for head h
        ldmatrix_x4(qb, qaddr[h] ^ (64u * (2 * i + gg)));
        const float(&nc)[2] = st.ncorr[2 * i + gg];
        const float seed[4] = {nc[0], nc[1], nc[0], nc[1]};
#pragma unroll
        for (int sub = 0; sub < 2; ++sub) {
          const uint32_t w0 = kr[2 * gg] >> (8 * sub), w1 = kr[2 * gg + 1] >> (8 * sub);
          const uint32_t a[4] = {int4_lo_biased(w0), int4_lo_biased(w1), int4_hi_biased(w0), int4_hi_biased(w1)};
          if (h == 0 && sub == 0)
            mma_16816(acc[gg], a, qb[0], qb[1], seed);
          else
            mma_16816(acc[gg], a, qb[2 * sub], qb[2 * sub + 1], acc[gg]);
        }
      }
    }
#pragma unroll
    for (int gg = 0; gg < 2; ++gg) {
      const int g = 2 * i + gg;
      if (g == 0) {
        s[0] = ks[0][g] * acc[gg][0];
        s[1] = ks[0][g] * acc[gg][1];
        s[2] = ks[1][g] * acc[gg][2];
        s[3] = ks[1][g] * acc[gg][3];
      } else {
        s[0] = fmaf(ks[0][g], acc[gg][0], s[0]);
        s[1] = fmaf(ks[0][g], acc[gg][1], s[1]);
        s[2] = fmaf(ks[1][g], acc[gg][2], s[2]);
        s[3] = fmaf(ks[1][g], acc[gg][3], s[3]);
      }
    }
  }
}

// O^T += V_h^T P'_h^T over the warp's heads for one page.  p[0..3] are the
// lane's probabilities in the score layout; vsc is the column of the lane's
// B-operand head (column g8) in the V scale block; tokens >= `valid` get a
// zero V scale when MASK.
template <int D, int HP, bool MASK>
IRIS_DEV void pair_page_pv(PairState<D>& st, uint32_t vstage, const uint32_t (&klane)[HP], uint32_t vsc,
                           int scale_stride, int valid, const float (&p)[4], int lane) {
  constexpr int G = D / 32;
  constexpr int CW = 8 / HP;
  const int t = lane & 3;
  const int hb = (lane >> 2) / CW;  // head of this lane's B column
  uint32_t sv01[G], sv89[G];
  {
    uint32_t raw[4][G / 2];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int tok = 2 * t + (k & 1) + 8 * (k >> 1);
      const uint32_t sp = vsc + tok * scale_stride;
      const bool ok = !MASK || tok < valid;
      if constexpr (G == 4) {
        const uint2 u = lds64(sp);
        raw[k][0] = ok ? u.x : 0u;
        raw[k][1] = ok ? u.y : 0u;
      } else {
        const uint32_t u = lds32(sp);
        raw[k][0] = ok ? u : 0u;
      }
    }
#pragma unroll
    for (int j = 0; j < G / 2; ++j) {
      sv01[2 * j] = prmt(raw[0][j], raw[1][j], 0x5410);
      sv01[2 * j + 1] = prmt(raw[0][j], raw[1][j], 0x7632);
      sv89[2 * j] = prmt(raw[2][j], raw[3][j], 0x5410);
      sv89[2 * j + 1] = prmt(raw[2][j], raw[3][j], 0x7632);
    }
  }
  const uint32_t pb0 = movmatrix_trans(h2_as_u32(__floats2half2_rn(p[0], p[1])));
  const uint32_t pb1 = movmatrix_trans(h2_as_u32(__floats2half2_rn(p[2], p[3])));
#pragma unroll
  for (int h = 0; h < HP; ++h) {
    const uint32_t q0 = hb == h ? pb0 : 0u, q1 = hb == h ? pb1 : 0u;
#pragma unroll
    for (int i = 0; i < G / 2; ++i) {
      uint32_t r[4];
      ldmatrix_x4_trans(r, (vstage + klane[h]) ^ (32u * i));
#pragma unroll
      for (int gg = 0; gg < 2; ++gg) {
        const int g = 2 * i + gg;
        const uint32_t wa = r[2 * gg], wb = r[2 * gg + 1];
        const uint32_t b0 = h2_as_u32(__hmul2(u32_as_h2(q0), u32_as_h2(sv01[g])));
        const uint32_t b1 = h2_as_u32(__hmul2(u32_as_h2(q1), u32_as_h2(sv89[g])));
#pragma unroll
        for (int jj = 0; jj < 2; ++jj) {
          const uint32_t xa = wa >> (8 * jj), xb = wb >> (8 * jj);
          const uint32_t a[4] = {int4_lo_exact(xa), int4_hi_exact(xa), int4_lo_exact(xb), int4_hi_exact(xb)};
          mma_16816(st.o[2 * g + jj], a, b0, b1, st.o[2 * g + jj]);
        }
      }
    }
  }
}

// One page with an online-softmax update whose running maximum may be stale
// by up to 8 (log2 units): y = scale*s - m is computed with one FFMA, and
// only when some y exceeds 8 (probabilities would pass 2^8) does the warp
// find the column maxima, raise m to them and rescale O and l.  Otherwise
// p = 2^y <= 256, still exact enough in fp16 for the PV product, and the
// max reduction and the rescale are skipped.  `first` marks a piece's first
// page: m then starts at that page's maxima (O and l are still zero).
template <int D, int HP, bool MASK>
IRIS_DEV void pair_process_page(PairState<D>& st, uint32_t base, const uint32_t (&klane)[HP], uint32_t v_off,
                                 const uint32_t (&qaddr)[HP], uint32_t ks_off, uint32_t vs_off, int scale_stride,
                                 int valid, float scale_log2, bool first, int lane) {
  const int g8 = lane >> 2;
  float s[4];
  pair_page_scores<D, HP>(st, base, klane, qaddr, base + ks_off, scale_stride, lane, s);
  float y[4];
  y[0] = fmaf(s[0], scale_log2, -st.m[0]);
  y[1] = fmaf(s[1], scale_log2, -st.m[1]);
  y[2] = fmaf(s[2], scale_log2, -st.m[0]);
  y[3] = fmaf(s[3], scale_log2, -st.m[1]);
  if (MASK) {
    if (g8 >= valid) y[0] = y[1] = kNegInf;
    if (g8 + 8 >= valid) y[2] = y[3] = kNegInf;
  }
  float mx0 = fmaxf(y[0], y[2]), mx1 = fmaxf(y[1], y[3]);
  if (__any_sync(0xffffffffu, first || fmaxf(mx0, mx1) > 8.0f)) {
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
    }
    // raise each column's maximum by inc (never lower it after the first page)
    const float inc0 = first ? mx0 : fmaxf(mx0, 0.f), inc1 = first ? mx1 : fmaxf(mx1, 0.f);
    st.m[0] += inc0;
    st.m[1] += inc1;
    y[0] -= inc0;
    y[1] -= inc1;
    y[2] -= inc0;
    y[3] -= inc1;
    if (!first) {
      const float c0 = ex2(-inc0), c1 = ex2(-inc1);
#pragma unroll
      for (int i = 0; i < D / 16; ++i) {
        st.o[i][0] *= c0;
        st.o[i][1] *= c1;
        st.o[i][2] *= c0;
        st.o[i][3] *= c1;
      }
      st.l[0] *= c0;
      st.l[1] *= c1;
    }
  }
  float pr[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) pr[k] = ex2(y[k]);  // ex2(-inf) = 0 for masked tokens
  st.l[0] += pr[0] + pr[2];
  st.l[1] += pr[1] + pr[3];
  pair_page_pv<D, HP, MASK>(st, base + v_off, klane, base + vs_off, scale_stride, valid, pr, lane);
}

// Finish a (sequence piece, head group): column c of the fragments is query
// head (kv0 + c / CW) * qpk + c % CW.
template <int D, int HP>
IRIS_DEV void pair_finish_piece(const DecodeParams& p, PairState<D>& st, int b, int kv0, bool complete, int64_t rec,
                                int lane) {
  constexpr int CW = 8 / HP;
  const int g8 = lane >> 2, t = lane & 3;
  float l0 = st.l[0], l1 = st.l[1];
#pragma unroll
  for (int o = 4; o < 32; o <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, o);
    l1 += __shfl_xor_sync(0xffffffffu, l1, o);
  }
  const float inv[2] = {1.0f / l0, 1.0f / l1};
  const float lse[2] = {st.m[0] + lg2(l0), st.m[1] + lg2(l1)};
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int c = 2 * t + j;
    if (c % CW >= p.qpk) continue;
    const int qh = (kv0 + c / CW) * p.qpk + c % CW;
#pragma unroll
    for (int g = 0; g < D / 32; ++g) {
      const float v0 = st.o[2 * g][j] * inv[j];
      const float v1 = st.o[2 * g][2 + j] * inv[j];
      const float v2 = st.o[2 * g + 1][j] * inv[j];
      const float v3 = st.o[2 * g + 1][2 + j] * inv[j];
      const int d = 32 * g + 4 * g8;
      if (complete && p.out_mode == IRIS_DECODE_OUT_FP16) {
        __half* dst = static_cast<__half*>(p.out) + (static_cast<int64_t>(b) * p.hq + qh) * D + d;
        uint2 u;
        u.x = h2_as_u32(__floats2half2_rn(v0, v1));
        u.y = h2_as_u32(__floats2half2_rn(v2, v3));
        *reinterpret_cast<uint2*>(dst) = u;
      } else {
        float* dst = complete ? static_cast<float*>(p.out) + (static_cast<int64_t>(b) * p.hq + qh) * D + d
                              : p.rec_o + (rec * p.hq + qh) * D + d;
        *reinterpret_cast<float4*>(dst) = make_float4(v0, v1, v2, v3);
      }
    }
    if (g8 == 0) {
      if (complete) {
        if (p.out_mode == IRIS_DECODE_OUT_LSE) p.out_lse[static_cast<int64_t>(b) * p.hq + qh] = lse[j];
      } else {
        p.rec_lse[rec * p.hq + qh] = lse[j];
      }
    }
  }
}

// Decode CTA with HB/HP consumer warps of HP heads each + 1 producer warp.
// Shared memory: the stage ring, the full/empty barriers, a 256-byte zero
// block, then one 2*8*D-byte query tile per consumer warp.
template <int D, int HP, bool R128>
__global__ void __maxnreg__(128) decode_pair_kernel(const __grid_constant__ CUtensorMap kmap,
                                                             const __grid_constant__ CUtensorMap vmap,
                                                             const DecodeParams p) {
  using C = DecCfg<D>;
  constexpr int CW = 8 / HP;
  grid_dependents_launch();  // the combine kernel may launch and wait meanwhile
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

  const int hblk = blockIdx.x;
  const int r = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int HB = p.hb;
  const int NW = HB / HP;  // consumer warps
  const int S = p.stages;
  __shared__ CtaPlan plan;

  const int scale_block = kPage * p.hkv * C::kGroups * 2;
  const int stage_bytes = ((2 * HB * C::kTileBytes + 2 * scale_block) + 1023) & ~1023;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * stage_bytes);
  uint64_t* empty = full + S;
  uint8_t* zero_blk = smem + ((S * stage_bytes + 16 * S + 255) & ~255);
  uint8_t* qtiles = zero_blk + 256;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, NW);
    }
    fence_barrier_init();
  }
  if (threadIdx.x < 64) reinterpret_cast<uint32_t*>(zero_blk)[threadIdx.x] = 0u;
  if (warp == 0) plan_cta(p, r, gridDim.y, blockIdx.x == 0 && r == 0, lane, &plan);
  __syncthreads();
  const int64_t U = plan.U;
  const int R = plan.R;
  if (r >= R) return;  // uniform per CTA (nothing was issued yet)

  const int64_t u0 = range_start(r, U, R), u1 = range_start(r + 1, U, R);
  const int b_first = plan.b_first;
  const int64_t ps_first = plan.ps_first;
  const uint32_t full_u32 = smem_u32(full), empty_u32 = smem_u32(empty);

  if (warp == NW) {
    run_producer<Int4Copy<R128 ? 256 / D : 1>, C::kTileBytes>(&kmap, &vmap, p, smem, stage_bytes, S, HB, hblk, u0,
                                                              u1, b_first, ps_first, full, full_u32, empty_u32,
                                                              scale_block, lane);
    return;
  }

  // ========================= consumer warps =========================
  const int kv0 = hblk * HB + warp * HP;  // first KV head of this warp
  const int g8 = lane >> 2, t = lane & 3;
  PairState<D> st;
  const uint32_t ring = smem_u32(smem);
  const uint32_t qtile = smem_u32(qtiles) + warp * (16 * D);
  // ldmatrix row addresses of the masked query tile per head: lane l reads
  // row (l & 7) of matrix (l >> 3); rows of other heads read the zero block
  uint32_t qaddr[HP];
  {
    const int row = lane & 7, x = (lane >> 3) ^ row;
#pragma unroll
    for (int h = 0; h < HP; ++h)
      qaddr[h] = (row / CW == h ? qtile + row * (2 * D) : smem_u32(zero_blk)) | (x << 4);
  }
  // this lane's ldmatrix addresses of the warp's heads, relative to a stage's K
  // region (the V region follows it at HB tiles)
  uint32_t klane[HP];
#pragma unroll
  for (int h = 0; h < HP; ++h) klane[h] = KvTiles<D, R128>::lane_off(lane, warp * HP + h);
  const uint32_t v_off = HB * C::kTileBytes;
  const uint32_t ks_off = 2 * HB * C::kTileBytes + (kv0 + (2 * t) / CW) * C::kGroups * 2;
  const uint32_t vs_off = 2 * HB * C::kTileBytes + scale_block + (kv0 + g8 / CW) * C::kGroups * 2;
  const int scale_stride = p.hkv * C::kGroups * 2;
  int s = 0;
  uint32_t ph = 0;
  uint32_t stage = ring;
  int b = b_first;
  int64_t ps = ps_first;  // first page of sequence b
  int64_t u = u0;
  while (u < u1) {
    const int64_t pe = ps + seq_pages(p, b);
    if (pe <= u) {
      ps = pe;
      ++b;
      continue;
    }
    const int64_t hi = pe < u1 ? pe : u1;
    const int L = min(p.seq_lens[b], p.max_pages * kPage);
    __syncwarp();  // the previous piece's ldmatrix reads of the tile are done
    pair_load_query<D, HP>(st, p.query + static_cast<int64_t>(b) * p.hq * D, kv0, p.qpk, qtile, lane);
    int valid = L - static_cast<int>(u - ps) * kPage;  // tokens left from this page on
    bool first = true;
    for (int64_t left = hi - u; left > 0; --left) {
      if (!mbar_wait_bounded(full_u32 + 8 * s, ph, p.err)) return;
      if (valid >= kPage)
        pair_process_page<D, HP, false>(st, stage, klane, v_off, qaddr, ks_off, vs_off, scale_stride, valid,
                                        p.scale_log2, first, lane);
      else
        pair_process_page<D, HP, true>(st, stage, klane, v_off, qaddr, ks_off, vs_off, scale_stride, valid,
                                       p.scale_log2, first, lane);
      __syncwarp();
      if (lane == 0) mbar_arrive(empty_u32 + 8 * s);
      first = false;
      valid -= kPage;
      if (++s == S) {
        s = 0;
        ph ^= 1;
        stage = ring;
      } else {
        stage += stage_bytes;
      }
    }
    const bool complete = (ps >= u0) && (pe <= u1);
    const int64_t rec = static_cast<int64_t>(r) * 2 + (u == u0 ? 0 : 1);
    pair_finish_piece<D, HP>(p, st, b, kv0, complete, rec, lane);
    u = hi;
    ps = pe;
    ++b;
  }
}

// ------------------------------------------------------- FP16 cache decode
// The matched FP16 baseline (reference fused_attention.py:223-370,528-582):
// k_cache / v_cache [pages, 16, Hkv, D] fp16.  Same split-KV schedule,
// producer and combine as the INT4 decode; a stage holds each head's K and V
// tile as [D/64 halves][16 tokens][128 bytes], 128-byte swizzled, so the
// consumer reads MMA fragments with ldmatrix (K) and ldmatrix.trans (V)
// without conversions.  One KV head per consumer warp, NT n-tiles of 8
// query heads.

template <int D>
struct Fp16Cfg {
  static constexpr int kTileBytes = kPage * D * 2;  // one head's K (or V) tile of a page
  static constexpr int kHalves = D / 64;            // 128-byte rows per token
};

template <int D, int NT>
struct Fp16State {
  float o[NT][D / 16][4];
  float m[NT][2];
  float l[NT][2];
  uint32_t qf[NT][D / 16][2];  // Q as mma B fragments
};

// Byte offset of 16-byte chunk `chunk` of token row `tok` in half `half` of a
// tile (128-byte swizzle: chunk index XOR token & 7).
IRIS_DEV uint32_t fp16_tile_off(int half, int tok, int chunk) {
  return (half * kPage + tok) * 128 + ((chunk ^ (tok & 7)) << 4);
}

template <int D, int NT>
IRIS_DEV void fp16_load_query(Fp16State<D, NT>& st, const __half* __restrict__ q_seq, int qpk, int lane) {
  const int n = lane >> 2, t = lane & 3;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int qh = nt * 8 + n;
    const __half* q = q_seq + qh * D;
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
      uint32_t b0 = 0, b1 = 0;
      if (qh < qpk) {
        b0 = *reinterpret_cast<const uint32_t*>(q + 16 * ks + 2 * t);
        b1 = *reinterpret_cast<const uint32_t*>(q + 16 * ks + 8 + 2 * t);
      }
      st.qf[nt][ks][0] = b0;
      st.qf[nt][ks][1] = b1;
    }
#pragma unroll
    for (int i = 0; i < D / 16; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) st.o[nt][i][j] = 0.f;
    st.m[nt][0] = st.m[nt][1] = 0.f;  // replaced by the first page's maxima
    st.l[nt][0] = st.l[nt][1] = 0.f;
  }
}

// One page of this warp's head: lazy online softmax as in pair_process_page.
// Tokens >= valid (MASK) are masked, and their V rows are zeroed in shared
// memory first (the cache may hold anything there, even NaN).
template <int D, int NT, bool MASK>
IRIS_DEV void fp16_process_page(Fp16State<D, NT>& st, uint32_t ktile, uint32_t vtile, uint8_t* vtile_ptr, int valid,
                                float scale_log2, bool first, int lane) {
  const int g8 = lane >> 2;
  const int mat = lane >> 3;
  // ---- scores: S^T[tok][qh] = K . Q^T, two accumulator chains ----
  float s[NT][4];
  {
    float acc[NT][2][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int c = 0; c < 2; ++c)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[nt][c][j] = 0.f;
    const int tok = (lane & 7) + 8 * (mat & 1);
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
      uint32_t a[4];
      ldmatrix_x4(a, ktile + fp16_tile_off(ks / 4, tok, 2 * (ks % 4) + (mat >> 1)));
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) mma_16816(acc[nt][ks & 1], a, st.qf[nt][ks][0], st.qf[nt][ks][1], acc[nt][ks & 1]);
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int j = 0; j < 4; ++j) s[nt][j] = acc[nt][0][j] + acc[nt][1][j];
  }
  if (MASK) {
    // zero the V rows of tokens past the end (lanes split the rows' 16-byte chunks)
    constexpr int kChunks = kPage * (D / 8);  // 16-byte chunks in a V tile
    for (int c = lane; c < kChunks; c += 32) {
      const int row = c / (D / 8);  // token
      if (row >= valid) {
        const int ch = c % (D / 8);
        *reinterpret_cast<uint4*>(vtile_ptr + fp16_tile_off(ch / 8, row, ch % 8)) = make_uint4(0, 0, 0, 0);
      }
    }
    fence_proxy_async_shared();
    __syncwarp();
  }
  float pr[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    float y[4];
    y[0] = fmaf(s[nt][0], scale_log2, -st.m[nt][0]);
    y[1] = fmaf(s[nt][1], scale_log2, -st.m[nt][1]);
    y[2] = fmaf(s[nt][2], scale_log2, -st.m[nt][0]);
    y[3] = fmaf(s[nt][3], scale_log2, -st.m[nt][1]);
    if (MASK) {
      if (g8 >= valid) y[0] = y[1] = kNegInf;
      if (g8 + 8 >= valid) y[2] = y[3] = kNegInf;
    }
    float mx0 = fmaxf(y[0], y[2]), mx1 = fmaxf(y[1], y[3]);
    if (__any_sync(0xffffffffu, first || fmaxf(mx0, mx1) > 8.0f)) {
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) {
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
      }
      const float inc0 = first ? mx0 : fmaxf(mx0, 0.f), inc1 = first ? mx1 : fmaxf(mx1, 0.f);
      st.m[nt][0] += inc0;
      st.m[nt][1] += inc1;
      y[0] -= inc0;
      y[1] -= inc1;
      y[2] -= inc0;
      y[3] -= inc1;
      if (!first) {
        const float c0 = ex2(-inc0), c1 = ex2(-inc1);
#pragma unroll
        for (int i = 0; i < D / 16; ++i) {
          st.o[nt][i][0] *= c0;
          st.o[nt][i][1] *= c1;
          st.o[nt][i][2] *= c0;
          st.o[nt][i][3] *= c1;
        }
        st.l[nt][0] *= c0;
        st.l[nt][1] *= c1;
      }
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) pr[nt][k] = ex2(y[k]);
    st.l[nt][0] += pr[nt][0] + pr[nt][2];
    st.l[nt][1] += pr[nt][1] + pr[nt][3];
  }
  // ---- O^T += V^T . P^T ----
  uint32_t pb[NT][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    pb[nt][0] = movmatrix_trans(h2_as_u32(__floats2half2_rn(pr[nt][0], pr[nt][1])));
    pb[nt][1] = movmatrix_trans(h2_as_u32(__floats2half2_rn(pr[nt][2], pr[nt][3])));
  }
  const int vtok = (lane & 7) + 8 * (mat >> 1);
#pragma unroll
  for (int i = 0; i < D / 16; ++i) {
    uint32_t a[4];
    ldmatrix_x4_trans(a, vtile + fp16_tile_off(i / 4, vtok, 2 * (i % 4) + (mat & 1)));
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) mma_16816(st.o[nt][i], a, pb[nt][0], pb[nt][1], st.o[nt][i]);
  }
}

// Output (or record) of a piece: O^T rows are head dims 16i + g8 (+8).
template <int D, int NT>
IRIS_DEV void fp16_finish_piece(const DecodeParams& p, Fp16State<D, NT>& st, int b, int kvh, bool complete,
                                int64_t rec, int lane) {
  const int g8 = lane >> 2, t = lane & 3;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    float l0 = st.l[nt][0], l1 = st.l[nt][1];
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      l0 += __shfl_xor_sync(0xffffffffu, l0, o);
      l1 += __shfl_xor_sync(0xffffffffu, l1, o);
    }
    const float inv[2] = {1.0f / l0, 1.0f / l1};
    const float lse[2] = {st.m[nt][0] + lg2(l0), st.m[nt][1] + lg2(l1)};
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int qh_local = nt * 8 + 2 * t + j;
      if (qh_local >= p.qpk) continue;
      const int qh = kvh * p.qpk + qh_local;
      const int64_t row = complete ? static_cast<int64_t>(b) * p.hq + qh : rec * p.hq + qh;
#pragma unroll
      for (int i = 0; i < D / 16; ++i) {
        const float v0 = st.o[nt][i][j] * inv[j], v1 = st.o[nt][i][2 + j] * inv[j];
        const int d = 16 * i + g8;
        if (complete && p.out_mode == IRIS_DECODE_OUT_FP16) {
          __half* dst = static_cast<__half*>(p.out) + row * D;
          dst[d] = __float2half_rn(v0);
          dst[d + 8] = __float2half_rn(v1);
        } else {
          float* dst = (complete ? static_cast<float*>(p.out) : p.rec_o) + row * D;
          dst[d] = v0;
          dst[d + 8] = v1;
        }
      }
      if (g8 == 0) {
        if (complete) {
          if (p.out_mode == IRIS_DECODE_OUT_LSE) p.out_lse[static_cast<int64_t>(b) * p.hq + qh] = lse[j];
        } else {
          p.rec_lse[rec * p.hq + qh] = lse[j];
        }
      }
    }
  }
}

template <int D, int NT>
__global__ void __maxnreg__(128) decode_fp16_kernel(const __grid_constant__ CUtensorMap kmap,
                                                            const __grid_constant__ CUtensorMap vmap,
                                                            const DecodeParams p) {
  using C = Fp16Cfg<D>;
  grid_dependents_launch();  // the combine kernel may launch and wait meanwhile
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

  const int hblk = blockIdx.x;
  const int r = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int HB = p.hb;
  const int S = p.stages;
  __shared__ CtaPlan plan;

  const int stage_bytes = (2 * HB * C::kTileBytes + 1023) & ~1023;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * stage_bytes);
  uint64_t* empty = full + S;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, HB);
    }
    fence_barrier_init();
  }
  if (warp == 0) plan_cta(p, r, gridDim.y, blockIdx.x == 0 && r == 0, lane, &plan);
  __syncthreads();
  const int64_t U = plan.U;
  const int R = plan.R;
  if (r >= R) return;  // uniform per CTA (nothing was issued yet)

  const int64_t u0 = range_start(r, U, R), u1 = range_start(r + 1, U, R);
  const int b_first = plan.b_first;
  const int64_t ps_first = plan.ps_first;
  const uint32_t full_u32 = smem_u32(full), empty_u32 = smem_u32(empty);

  if (warp == HB) {
    run_producer<Fp16Copy<(D > 64) ? 5 : 4>, C::kTileBytes>(&kmap, &vmap, p, smem, stage_bytes, S, HB, hblk, u0, u1,
                                                            b_first, ps_first, full, full_u32, empty_u32, 0, lane);
    return;
  }

  // ========================= consumer warps =========================
  const int kvh = hblk * HB + warp;
  Fp16State<D, NT> st;
  const uint32_t ring = smem_u32(smem);
  const uint32_t k_off = warp * C::kTileBytes, v_off = (HB + warp) * C::kTileBytes;
  int s = 0;
  uint32_t ph = 0;
  uint32_t stage = ring;
  uint8_t* stage_ptr = smem;
  int b = b_first;
  int64_t ps = ps_first;
  int64_t u = u0;
  while (u < u1) {
    const int64_t pe = ps + seq_pages(p, b);
    if (pe <= u) {
      ps = pe;
      ++b;
      continue;
    }
    const int64_t hi = pe < u1 ? pe : u1;
    const int L = min(p.seq_lens[b], p.max_pages * kPage);
    fp16_load_query<D, NT>(st, p.query + (static_cast<int64_t>(b) * p.hq + kvh * p.qpk) * D, p.qpk, lane);
    int valid = L - static_cast<int>(u - ps) * kPage;
    bool first = true;
    for (int64_t left = hi - u; left > 0; --left) {
      if (!mbar_wait_bounded(full_u32 + 8 * s, ph, p.err)) return;
      if (valid >= kPage)
        fp16_process_page<D, NT, false>(st, stage + k_off, stage + v_off, stage_ptr + v_off, valid, p.scale_log2,
                                        first, lane);
      else
        fp16_process_page<D, NT, true>(st, stage + k_off, stage + v_off, stage_ptr + v_off, valid, p.scale_log2,
                                       first, lane);
      __syncwarp();
      if (lane == 0) mbar_arrive(empty_u32 + 8 * s);
      first = false;
      valid -= kPage;
      if (++s == S) {
        s = 0;
        ph ^= 1;
        stage = ring;
        stage_ptr = smem;
      } else {
        stage += stage_bytes;
        stage_ptr += stage_bytes;
      }
    }
    const bool complete = (ps >= u0) && (pe <= u1);
    const int64_t rec = static_cast<int64_t>(r) * 2 + (u == u0 ? 0 : 1);
    fp16_finish_piece<D, NT>(p, st, b, kvh, complete, rec, lane);
    u = hi;
    ps = pe;
    ++b;
  }
}

// ---------------------------------------------------------- combine kernel
// Grid (sequence, share): the CTAs of a sequence split its (query head,
// 4 dims) items, so many SMs take part.  An item merges the records of the
// ranges the sequence touches (record k: the first range's record, then
// side 0 of each later range), eight per load round with an online rescale,
// spread over combine_lanes adjacent lanes when a sequence spans many
// ranges.  Sequences finished inside one range were written by the decode
// kernel and are skipped.
constexpr int kCombineThreads = 256;

// Where sequence b's pages sit in the batch's concatenation, the total U and
// the ranges R in use, recomputed from seq_lens exactly as the decode's plan
// computes them (an input of the call, so this runs while the decode is
// still working): warp 0 of the CTA, the result in shared memory.
struct SeqSpan {
  int64_t ps, pe, U;
  int32_t R;
};

IRIS_DEV void combine_span(const DecodeParams& p, int b, int lane, SeqSpan* out) {
  int64_t U = 0, ps = 0, pe = 0;
  for (int base = 0; base < p.batch; base += 32) {
    const int bb = base + lane;
    int32_t np = bb < p.batch ? seq_pages(p, bb) : 0;
    int32_t x = np;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int32_t y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (bb == b) {
      ps = U + x - np;
      pe = U + x;
    }
    U += __shfl_sync(0xffffffffu, x, 31);
  }
  const int src = b & 31;
  ps = __shfl_sync(0xffffffffu, ps, src);
  pe = __shfl_sync(0xffffffffu, pe, src);
  int32_t R = 0;
  if (U > 0) {
    const int64_t want = wanted_ranges(U);
    R = static_cast<int32_t>(want < p.ranges ? want : p.ranges);
  }
  if (lane == 0) *out = SeqSpan{ps, pe, U, R};
}

template <int D>
__global__ void __launch_bounds__(kCombineThreads) decode_combine_kernel(const DecodeParams p) {
  const int b = blockIdx.x;
  __shared__ SeqSpan span;
  if (threadIdx.x < 32) combine_span(p, b, threadIdx.x, &span);
  __syncthreads();
  const int64_t U = span.U, R = span.R;
  const int64_t ps = span.ps, pe = span.pe;
  if (pe <= ps) return;
  const int64_t f = range_of_page(ps, U, R), l = range_of_page(pe - 1, U, R);
  if (f == l) return;  // finished inside one range by the decode kernel
  grid_dependency_wait();  // the records come from the decode kernel
  const int n = static_cast<int>(l - f + 1);
  const int64_t rec_first = f * 2 + (ps > range_start(f, U, R) ? 1 : 0);
  constexpr int kQuads = D / 4;
  // T lanes of a warp share one (query head, 4 dims) item: lane j of the
  // group merges records j, j + T, j + 2T, ... (eight per load round), then
  // the group combines its partial merges with shuffles.  Sequences split
  // over many ranges (small batches) thus need one or two load rounds, not
  // n / 8.  A warp holds G = 32 / T items and the lanes of one item are G
  // apart, so the G lanes of each record's load read adjacent quads of one
  // record (G * 16 contiguous bytes).
  const int T = p.combine_lanes;
  const int G = 32 / T;
  const int items = p.hq * kQuads;
  const int lane = threadIdx.x & 31;
  const int item = ((blockIdx.y * blockDim.x + threadIdx.x) >> 5) * G + lane % G, j = lane / G;
  const bool valid = item < items;
  const int qh = item / kQuads, t = item % kQuads;
  float m = kNegInf, wsum = 0.f;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  if (valid) {
    for (int k0 = j; k0 < n; k0 += 8 * T) {
      float lse[8];
      float4 o[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int k = k0 + i * T;
        if (k < n) {
          const int64_t rec = k == 0 ? rec_first : (f + k) * 2;
          lse[i] = p.rec_lse[rec * p.hq + qh];
          o[i] = *reinterpret_cast<const float4*>(p.rec_o + (rec * p.hq + qh) * D + 4 * t);
        } else {
          lse[i] = kNegInf;
          o[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
      float mc = m;
#pragma unroll
      for (int i = 0; i < 8; ++i) mc = fmaxf(mc, lse[i]);
      const float c = ex2(m - mc);  // rescale of what was merged so far (0 on the first chunk)
      acc.x *= c;
      acc.y *= c;
      acc.z *= c;
      acc.w *= c;
      wsum *= c;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float w = ex2(lse[i] - mc);  // 0 for padding
        acc.x = fmaf(w, o[i].x, acc.x);
        acc.y = fmaf(w, o[i].y, acc.y);
        acc.z = fmaf(w, o[i].z, acc.z);
        acc.w = fmaf(w, o[i].w, acc.w);
        wsum += w;
      }
      m = mc;
    }
  }
  // combine the group's partial merges (its lanes are G apart)
  for (int o = G; o < 32; o <<= 1) {
    const float mo = __shfl_xor_sync(0xffffffffu, m, o);
    const float wo = __shfl_xor_sync(0xffffffffu, wsum, o);
    const float ax = __shfl_xor_sync(0xffffffffu, acc.x, o), ay = __shfl_xor_sync(0xffffffffu, acc.y, o);
    const float az = __shfl_xor_sync(0xffffffffu, acc.z, o), aw = __shfl_xor_sync(0xffffffffu, acc.w, o);
    const float mn = fmaxf(m, mo);
    const float cs = mn == kNegInf ? 0.f : ex2(m - mn), co = mn == kNegInf ? 0.f : ex2(mo - mn);
    acc.x = acc.x * cs + ax * co;
    acc.y = acc.y * cs + ay * co;
    acc.z = acc.z * cs + az * co;
    acc.w = acc.w * cs + aw * co;
    wsum = wsum * cs + wo * co;
    m = mn;
  }
  if (valid && j == 0) {
    const float inv = 1.0f / wsum;
    const int64_t orow = static_cast<int64_t>(b) * p.hq + qh;
    if (p.out_mode == IRIS_DECODE_OUT_FP16) {
      uint2 u;
      u.x = h2_as_u32(__floats2half2_rn(acc.x * inv, acc.y * inv));
      u.y = h2_as_u32(__floats2half2_rn(acc.z * inv, acc.w * inv));
      *reinterpret_cast<uint2*>(static_cast<__half*>(p.out) + orow * D + 4 * t) = u;
    } else {
      *reinterpret_cast<float4*>(static_cast<float*>(p.out) + orow * D + 4 * t) =
          make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
      if (t == 0) p.out_lse[orow] = m + lg2(wsum);
    }
  }
}

// Merge of log-sum-exp partials from several producers (e.g. GPUs).  Part k
// of row r: O at parts_o[k * o_stride + r * head_dim], lse at
// parts_lse[k * lse_stride + r].  A part with lse = -inf holds none of the
// row's tokens (a GPU without a split of that sequence) and is skipped, so
// its O may be left unwritten.
__global__ void merge_lse_kernel(const float* __restrict__ parts_o, const float* __restrict__ parts_lse,
                                 int32_t num_parts, int64_t rows, int32_t head_dim, int64_t o_stride,
                                 int64_t lse_stride, __half* __restrict__ out) {
  const int64_t row = blockIdx.x;
  if (row >= rows) return;
  float mx = kNegInf;
  for (int k = 0; k < num_parts; ++k) mx = fmaxf(mx, parts_lse[k * lse_stride + row]);
  for (int d = threadIdx.x; d < head_dim; d += blockDim.x) {
    float acc = 0.f, ws = 0.f;
    for (int k = 0; k < num_parts; ++k) {
      const float lse = parts_lse[k * lse_stride + row];
      if (lse == kNegInf) continue;
      const float w = ex2(lse - mx);
      acc = fmaf(w, parts_o[k * o_stride + row * head_dim + d], acc);
      ws += w;
    }
    out[row * head_dim + d] = __float2half_rn(acc / ws);
  }
}

}  // namespace iris

using namespace iris;

// ------------------------------------------------------------- host side

namespace {

constexpr int kSmemBudgetPerSm = 200 * 1024;

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// 4-D view of k_data / v_data: (D/2 bytes, 16 tokens of a page, Hkv heads,
// pages) with the token stride (Hkv*D/2) above the head stride (D/2).  A
// box of (D/2, 16, hb, 1) lands as hb per-head [16][D/2] tiles, swizzled so
// that ldmatrix reads them without bank conflicts: one copy per page per
// tensor for the whole head block.
//
// r128: the view (128 bytes, 16 tokens, Hkv / RH units, pages) with RH =
// 256 / D adjacent heads per 128-byte row and the 128-byte swizzle; a box of
// (128, 16, hb / RH, 1) lands as hb / RH tiles [16][128 B].
bool make_kv_map(CUtensorMap* map, const void* base, int D, int hkv, int hb, int64_t num_pages, bool r128) {
  EncodeTiledFn enc = encode_fn();
  if (enc == nullptr) return false;
  if (r128) {
    const int rh = 256 / D;
    const cuuint64_t dims[4] = {128u, static_cast<cuuint64_t>(kPage), static_cast<cuuint64_t>(hkv / rh),
                                static_cast<cuuint64_t>(num_pages)};
    const cuuint64_t strides[3] = {static_cast<cuuint64_t>(hkv) * (D / 2), 128u,
                                   static_cast<cuuint64_t>(hkv) * (D / 2) * kPage};
    const cuuint32_t box[4] = {128u, static_cast<cuuint32_t>(kPage), static_cast<cuuint32_t>(hb / rh), 1u};
    const cuuint32_t estr[4] = {1u, 1u, 1u, 1u};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<void*>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
  }
  const cuuint64_t dims[4] = {static_cast<cuuint64_t>(D / 2), static_cast<cuuint64_t>(kPage),
                              static_cast<cuuint64_t>(hkv), static_cast<cuuint64_t>(num_pages)};
  const cuuint64_t strides[3] = {static_cast<cuuint64_t>(hkv) * (D / 2), static_cast<cuuint64_t>(D / 2),
                                 static_cast<cuuint64_t>(hkv) * (D / 2) * kPage};
  const cuuint32_t box[4] = {static_cast<cuuint32_t>(D / 2), static_cast<cuuint32_t>(kPage),
                             static_cast<cuuint32_t>(hb), 1u};
  const cuuint32_t estr[4] = {1u, 1u, 1u, 1u};
  const CUtensorMapSwizzle sw = (D == 128) ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B;
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// FP16 cache [pages, 16, Hkv, D] fp16 viewed as (64 elements, 16 tokens,
// D/64 halves, Hkv heads, pages) with 128-byte swizzle: a box of (64, 16,
// D/64, hb, 1) lands as hb per-head tiles [D/64][16][128 B] (4-D without the
// halves dimension at D = 64).
bool make_fp16_map(CUtensorMap* map, const void* base, int D, int hkv, int hb, int64_t num_pages) {
  EncodeTiledFn enc = encode_fn();
  if (enc == nullptr) return false;
  const cuuint64_t row = static_cast<cuuint64_t>(hkv) * D * 2;  // bytes per token (all heads)
  const cuuint32_t estr[5] = {1u, 1u, 1u, 1u, 1u};
  if (D == 128) {
    const cuuint64_t dims[5] = {64u, static_cast<cuuint64_t>(kPage), 2u, static_cast<cuuint64_t>(hkv),
                                static_cast<cuuint64_t>(num_pages)};
    const cuuint64_t strides[4] = {row, 128u, static_cast<cuuint64_t>(D) * 2, row * kPage};
    const cuuint32_t box[5] = {64u, static_cast<cuuint32_t>(kPage), 2u, static_cast<cuuint32_t>(hb), 1u};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 5, const_cast<void*>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
  }
  const cuuint64_t dims[4] = {64u, static_cast<cuuint64_t>(kPage), static_cast<cuuint64_t>(hkv),
                              static_cast<cuuint64_t>(num_pages)};
  const cuuint64_t strides[3] = {row, static_cast<cuuint64_t>(D) * 2, row * kPage};
  const cuuint32_t box[4] = {64u, static_cast<cuuint32_t>(kPage), static_cast<cuuint32_t>(hb), 1u};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Tensor maps are pure functions of (format, base, D, Hkv, head block, pages); the
// last few are kept so that a decode loop over the same cache does not
// re-encode them on every call.
bool cached_kv_map(CUtensorMap* map, int fmt, const void* base, int D, int hkv, int hb, int64_t num_pages) {
  struct Entry {
    const void* base;
    int fmt, D, hkv, hb;
    int64_t pages;
    CUtensorMap map;
  };
  constexpr int kEntries = 16;
  static Entry cache[kEntries];
  static int used = 0, next = 0;
  static std::mutex mu;
  {
    std::lock_guard<std::mutex> lock(mu);
    for (int i = 0; i < used; ++i) {
      const Entry& e = cache[i];
      if (e.base == base && e.fmt == fmt && e.D == D && e.hkv == hkv && e.hb == hb && e.pages == num_pages) {
        *map = e.map;
        return true;
      }
    }
  }
  // fmt: 0 INT4 one head per row, 2 INT4 128-byte rows, 1 FP16
  if (!(fmt == 1 ? make_fp16_map(map, base, D, hkv, hb, num_pages)
                 : make_kv_map(map, base, D, hkv, hb, num_pages, fmt == 2)))
    return false;
  std::lock_guard<std::mutex> lock(mu);
  Entry& e = cache[next];
  e = Entry{base, fmt, D, hkv, hb, num_pages, *map};
  next = (next + 1) % kEntries;
  if (used < kEntries) ++used;
  return true;
}

using DecodeKernelFn = void (*)(CUtensorMap, CUtensorMap, DecodeParams);

// KV heads per consumer warp: groups of at most 4 query heads share a warp's
// 8 MMA columns between 2 (3-4 query heads) or 4 (1-2) KV heads
// (decode_pair_kernel); larger groups get one KV head per warp
// (decode_kernel).
int heads_per_warp(int qpk, int hkv) {
  if (qpk > 4) return 1;
  int hp = qpk <= 2 ? 4 : 2;
  while (hp > 1 && hkv % hp != 0) hp >>= 1;
  return hp;
}

// Cap on KV heads per CTA.  IRIS_DECODE_MAX_HB (1, 2, 4 or 8) overrides the
// defaults (8 with head groups per warp, else 4) for tuning.
int max_hb(int dflt) {
  static int v = [] {
    const char* e = getenv("IRIS_DECODE_MAX_HB");
    int x = e ? atoi(e) : 0;
    return (x == 1 || x == 2 || x == 4 || x == 8) ? x : 0;
  }();
  return v ? v : dflt;
}

// 128-byte-row tiles unless IRIS_DECODE_R128=0 (the one-head-per-row form,
// kept for comparison).
bool use_r128() {
  static const bool v = [] {
    const char* e = getenv("IRIS_DECODE_R128");
    return !(e && e[0] == '0');
  }();
  return v;
}

// The CTA shape of one decode problem.
struct Plan {
  DecodeKernelFn fn;
  int fp16;  // FP16 cache (decode_fp16_kernel): bigger tiles, no scale blocks
  int r128;  // INT4 tiles of 128-byte rows (head blocks of whole rows of 256 / D heads)
  int hp;    // KV heads per consumer warp
  int hb;    // KV heads per CTA (one TMA box)
  int nw;    // consumer warps = hb / hp
  int pair;  // decode_pair_kernel (query tiles in shared memory)
};

Plan make_plan(int D, int qpk, int hkv) {
  Plan pl;
  pl.fp16 = 0;
  pl.hp = heads_per_warp(qpk, hkv);
  pl.pair = pl.hp > 1;
  const int cap = max_hb(pl.pair ? 8 : 4);
  pl.hb = pl.hp;
  for (int hb = cap; hb >= pl.hp; hb >>= 1)
    if (hkv % hb == 0 && hb % pl.hp == 0) {
      pl.hb = hb;
      break;
    }
  pl.nw = pl.hb / pl.hp;
  pl.r128 = use_r128() && pl.hb % (256 / D) == 0;
  if (D == 128) {
    if (pl.r128)
      pl.fn = pl.hp == 4 ? decode_pair_kernel<128, 4, true> : pl.hp == 2 ? decode_pair_kernel<128, 2, true>
            : qpk <= 8   ? decode_kernel<128, 1, true>      : decode_kernel<128, 2, true>;
    else
      pl.fn = pl.hp == 4 ? decode_pair_kernel<128, 4, false> : pl.hp == 2 ? decode_pair_kernel<128, 2, false>
            : qpk <= 8   ? decode_kernel<128, 1, false>      : decode_kernel<128, 2, false>;
  } else {
    if (pl.r128)
      pl.fn = pl.hp == 4 ? decode_pair_kernel<64, 4, true> : pl.hp == 2 ? decode_pair_kernel<64, 2, true>
            : qpk <= 8   ? decode_kernel<64, 1, true>      : decode_kernel<64, 2, true>;
    else
      pl.fn = pl.hp == 4 ? decode_pair_kernel<64, 4, false> : pl.hp == 2 ? decode_pair_kernel<64, 2, false>
            : qpk <= 8   ? decode_kernel<64, 1, false>      : decode_kernel<64, 2, false>;
  }
  return pl;
}

struct LaunchShape {
  int stages, stage_bytes, smem, ranges, max_ranges;
};

// FP16 cache: one KV head per consumer warp, at most 4 heads per CTA (a
// stage holds 2 * 4 KB per head at D = 128).
Plan make_plan_fp16(int D, int qpk, int hkv) {
  Plan pl;
  pl.fp16 = 1;
  pl.r128 = 0;
  pl.hp = 1;
  pl.pair = 0;
  const int cap = max_hb(4);
  pl.hb = 1;
  for (int hb = cap; hb >= 1; hb >>= 1)
    if (hkv % hb == 0) {
      pl.hb = hb;
      break;
    }
  pl.nw = pl.hb;
  if (D == 128)
    pl.fn = qpk <= 8 ? decode_fp16_kernel<128, 1> : decode_fp16_kernel<128, 2>;
  else
    pl.fn = qpk <= 8 ? decode_fp16_kernel<64, 1> : decode_fp16_kernel<64, 2>;
  return pl;
}

int stage_bytes_fp16(int D, int hb) { return (2 * hb * kPage * D * 2 + 1023) & ~1023; }

int stage_bytes_for(int D, int hkv, int hb) {
  const int tile = kPage * D / 2;
  const int scale_block = kPage * hkv * (D / 32) * 2;
  return ((2 * hb * tile + 2 * scale_block) + 1023) & ~1023;
}

// Ring + barriers (+ zero block and query tiles for the pair kernel) + the
// slack for aligning the dynamic shared memory base to 1 KB.
int smem_for(const Plan& pl, int D, int stages, int stage_bytes) {
  int bytes = stages * stage_bytes + 2 * stages * 8;
  if (pl.pair) bytes = ((bytes + 255) & ~255) + 256 + pl.nw * 16 * D;
  return bytes + 1024;
}

int device_sms(int device) {
  static std::mutex mu;
  static std::map<int, int> cache;
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(device);
  if (it != cache.end()) return it->second;
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || sms <= 0) {
    cudaGetLastError();
    return 148;  // not cached: no device visible (host-only use)
  }
  cache[device] = sms;
  return sms;
}

int target_ctas_per_sm(const Plan& pl) { return 16 / pl.nw < 1 ? 1 : 16 / pl.nw; }

// Upper bound on the number of ranges (sizes the workspace): at most 16
// consumer warps' worth of CTAs per SM.
int max_ranges_for(int qpk, int hkv, int sms, bool fp16 = false) {
  const Plan pl = fp16 ? make_plan_fp16(128, qpk, hkv) : make_plan(128, qpk, hkv);
  const int r = sms * target_ctas_per_sm(pl) / (hkv / pl.hb);
  return r < 1 ? 1 : r;
}

// The dynamic shared memory limit is a per-kernel attribute shared by every
// shape, so it only ever grows (a smaller shape must not lower it under a
// larger cached one).
cudaError_t ensure_smem_attr(DecodeKernelFn fn, int device, int smem) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, int> set_to;
  std::lock_guard<std::mutex> lock(mu);
  int& cur = set_to[std::make_pair(reinterpret_cast<const void*>(fn), device)];
  if (smem <= cur) return cudaSuccess;
  const cudaError_t e = cudaFuncSetAttribute(reinterpret_cast<const void*>(fn),
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e == cudaSuccess) cur = smem;
  return e;
}

// Computed once per (kernel, Hkv, device): later calls make no attribute or
// occupancy queries, so the entry point can be captured in a CUDA graph
// after its first (uncaptured) call.
LaunchShape compute_launch_shape(const Plan& pl, int D, int qpk, int hkv, int device) {
  LaunchShape s;
  const int sms = device_sms(device);
  const int nhb = hkv / pl.hb;
  s.stage_bytes = pl.fp16 ? stage_bytes_fp16(D, pl.hb) : stage_bytes_for(D, hkv, pl.hb);
  s.max_ranges = max_ranges_for(qpk, hkv, sms, pl.fp16 != 0);
  const int threads = (pl.nw + 1) * 32;
  for (int target = target_ctas_per_sm(pl); target >= 1; --target) {
    const int fixed = smem_for(pl, D, 0, s.stage_bytes);
    int stages = (kSmemBudgetPerSm / target - fixed - 256) / (s.stage_bytes + 16);
    stages = stages < 2 ? 2 : (stages > 10 ? 10 : stages);
    const int smem = smem_for(pl, D, stages, s.stage_bytes);
    int occ = 0;
    if (ensure_smem_attr(pl.fn, device, smem) != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, reinterpret_cast<const void*>(pl.fn), threads, smem) !=
            cudaSuccess) {
      cudaGetLastError();
      occ = 0;
    }
    if (occ >= target || target == 1) {
      s.stages = stages;
      s.smem = smem;
      int ranges = sms * (occ < target ? (occ > 0 ? occ : 1) : target) / nhb;
      ranges = ranges < 1 ? 1 : ranges;
      s.ranges = ranges > s.max_ranges ? s.max_ranges : ranges;
      break;
    }
  }
  return s;
}

LaunchShape launch_shape(const Plan& pl, int D, int qpk, int hkv, int device) {
  static std::mutex mu;
  static std::map<std::tuple<const void*, int, int>, LaunchShape> cache;
  std::lock_guard<std::mutex> lock(mu);
  const auto key = std::make_tuple(reinterpret_cast<const void*>(pl.fn), hkv, device);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  const LaunchShape s = compute_launch_shape(pl, D, qpk, hkv, device);
  cache[key] = s;
  return s;
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

struct Workspace {
  int32_t* prefix;
  int32_t* meta;
  float* rec_lse;
  float* rec_o;
  size_t bytes;
};

Workspace carve(void* base, int batch, int hq, int D, int ranges) {
  Workspace w;
  uint8_t* p = static_cast<uint8_t*>(base);
  size_t off = 0;
  w.prefix = reinterpret_cast<int32_t*>(p + off);
  off += align256(sizeof(int32_t) * (batch + 1));
  w.meta = reinterpret_cast<int32_t*>(p + off);
  off += 256;
  w.rec_lse = reinterpret_cast<float*>(p + off);
  off += align256(sizeof(float) * 2 * static_cast<size_t>(ranges) * hq);
  w.rec_o = reinterpret_cast<float*>(p + off);
  off += align256(sizeof(float) * 2 * static_cast<size_t>(ranges) * hq * D);
  w.bytes = off;
  return w;
}

template <int D>
cudaError_t launch_decode(const Plan& pl, const CUtensorMap& km, const CUtensorMap& vm, DecodeParams p, int device,
                          cudaStream_t stream, int32_t ranges_cap) {
  const LaunchShape ls = launch_shape(pl, D, p.qpk, p.hkv, device);
  p.hb = pl.hb;
  p.stages = ls.stages;
  const int32_t ranges = ls.ranges < ranges_cap ? ls.ranges : ranges_cap;
  cudaError_t e;
  e = ensure_smem_attr(pl.fn, device, ls.smem);  // no-op once raised
  if (e != cudaSuccess) {
    record_cuda_error(e, "cudaFuncSetAttribute(max dynamic smem)");
    return e;
  }
  // head blocks of one range are adjacent in launch order: they share the
  // page's scale sectors and DRAM rows
  p.ranges = ranges;
  dim3 grid(p.hkv / pl.hb, ranges);
  pl.fn<<<grid, (pl.nw + 1) * 32, ls.smem, stream>>>(km, vm, p);
  e = cudaGetLastError();
  if (e != cudaSuccess) {
    record_cuda_error(e, "decode_kernel launch");
    return e;
  }
  // programmatic launch: the combine CTAs are resident before the decode ends
  // lanes per output item: enough that each merges at most ~8 records in one
  // load round (a sequence spans up to about ranges / batch + 2 ranges).  The
  // estimate uses the device's range count, not the problem-capped grid: the
  // lane count sets the merge order, so the output does not depend on the
  // block table's width
  const int rec_est = ls.ranges / p.batch + 2;
  int lanes = 1;
  while (lanes < 8 && (rec_est + lanes - 1) / lanes > 8) lanes <<= 1;
  p.combine_lanes = lanes;
  const int slots = p.hq * (D / 4) * lanes;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.batch, (slots + kCombineThreads - 1) / kCombineThreads);
  cfg.blockDim = dim3(kCombineThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, decode_combine_kernel<D>, p);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) record_cuda_error(e, "decode_combine_kernel launch");
  return e;
}

}  // namespace

// Page ranges a problem can use at most: a batch holds at most
// batch * max_pages_per_seq pages, and for every U <= pages wanted_ranges(U)
// is at most the largest of its three tiers' values at their largest U.
int32_t problem_ranges(int32_t batch, int32_t max_pages_per_seq) {
  const int64_t pages = static_cast<int64_t>(batch) * (max_pages_per_seq > 0 ? max_pages_per_seq : 1);
  const int64_t one = pages < kOnePageRanges ? pages : kOnePageRanges;
  const int64_t two = ((pages < kTwoPageRanges ? pages : kTwoPageRanges) + 1) / 2;
  const int64_t four = (pages + kMinPagesPerRange - 1) / kMinPagesPerRange;
  int64_t r = one > two ? one : two;
  r = r > four ? r : four;
  return static_cast<int32_t>(r < 1 ? 1 : (r > 0x7fffffff ? 0x7fffffff : r));
}

// Workspace bytes of a decode whose page ranges are capped by the problem
// (the allocation-free entry point carves its fixed array this way).
size_t problem_workspace_bytes(int32_t batch, int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                               int32_t max_pages_per_seq, int32_t device) {
  if (batch <= 0 || num_q_heads <= 0 || num_kv_heads <= 0 || (head_dim != 64 && head_dim != 128)) return 0;
  if (num_q_heads % num_kv_heads != 0) return 0;
  int32_t r = max_ranges_for(num_q_heads / num_kv_heads, num_kv_heads, device_sms(device));
  const int32_t cap = problem_ranges(batch, max_pages_per_seq);
  return carve(nullptr, batch, num_q_heads, head_dim, cap < r ? cap : r).bytes;
}

extern "C" size_t iris_b200_decode_workspace_bytes(int32_t batch, int32_t num_q_heads, int32_t num_kv_heads,
                                                   int32_t head_dim, int32_t device) {
  if (batch <= 0 || num_q_heads <= 0 || num_kv_heads <= 0 || (head_dim != 64 && head_dim != 128)) return 0;
  if (num_q_heads % num_kv_heads != 0) return 0;
  return carve(nullptr, batch, num_q_heads, head_dim,
               max_ranges_for(num_q_heads / num_kv_heads, num_kv_heads, device_sms(device)))
      .bytes;
}

// ranges_limit > 0 caps the page ranges (and so the workspace carve) below the
// SM-derived maximum; 0 keeps the maximum.
static int decode_entry(bool fp16, const void* query, const void* k_data, const void* v_data,
                        const void* k_scale, const void* v_scale, const int32_t* block_table,
                        int64_t block_table_stride, const int32_t* seq_lens, void* output, float* out_lse,
                        int32_t out_mode, int32_t batch, int32_t num_q_heads, int32_t num_kv_heads,
                        int32_t head_dim, int64_t num_pages, int32_t page_size, int32_t max_pages_per_seq,
                        float softmax_scale, void* workspace, size_t workspace_bytes, int32_t* error_word,
                        void* stream, int32_t ranges_limit = 0) {
  if (batch < 0 || num_q_heads <= 0 || num_kv_heads <= 0 || num_pages <= 0 || max_pages_per_seq < 0)
    return IRIS_EINVAL;
  if (page_size != kPage || (head_dim != 64 && head_dim != 128)) return IRIS_EUNSUPPORTED;
  if (num_q_heads % num_kv_heads != 0) return IRIS_EINVAL;
  const int qpk = num_q_heads / num_kv_heads;
  if (qpk > 16) return IRIS_EUNSUPPORTED;
  if (out_mode != IRIS_DECODE_OUT_FP16 && out_mode != IRIS_DECODE_OUT_LSE) return IRIS_EINVAL;
  if (batch == 0) return IRIS_OK;
  if (max_pages_per_seq > 0 && block_table_stride < max_pages_per_seq) return IRIS_EINVAL;
  const void* ptrs[] = {query, k_data, v_data, seq_lens, output, workspace, error_word};
  for (const void* q : ptrs)
    if (q == nullptr) return IRIS_EINVAL;
  if (!fp16 && (k_scale == nullptr || v_scale == nullptr)) return IRIS_EINVAL;
  if (max_pages_per_seq > 0 && block_table == nullptr) return IRIS_EINVAL;
  if (out_mode == IRIS_DECODE_OUT_LSE && out_lse == nullptr) return IRIS_EINVAL;
  if (!(softmax_scale > 0.0f) && !(softmax_scale < 0.0f)) return IRIS_EINVAL;
  auto al = [](const void* q, uintptr_t a) { return reinterpret_cast<uintptr_t>(q) % a == 0; };
  if (!al(k_data, 16) || !al(v_data, 16) || (!fp16 && (!al(k_scale, 16) || !al(v_scale, 16))) || !al(query, 16) ||
      !al(output, 16) || !al(workspace, 256))
    return IRIS_EALIGN;

  clear_stale_cuda_error();
  int device = 0;
  if (cudaError_t e0 = cudaGetDevice(&device); e0 != cudaSuccess) {
    record_cuda_error(e0, "cudaGetDevice");
    return IRIS_ECUDA;
  }
  int32_t max_ranges = max_ranges_for(qpk, num_kv_heads, device_sms(device), fp16);
  // a batch holds at most batch * max_pages_per_seq pages, so the plan never
  // cuts more ranges than problem_ranges: a small problem launches only the
  // CTAs it can use (the range boundaries, and so the results, are the same)
  const int32_t pcap = problem_ranges(batch, max_pages_per_seq);
  if (pcap < max_ranges) max_ranges = pcap;
  if (ranges_limit > 0 && ranges_limit < max_ranges) max_ranges = ranges_limit;
  const Workspace ws = carve(workspace, batch, num_q_heads, head_dim, max_ranges);
  if (workspace_bytes < ws.bytes) return IRIS_EWORKSPACE;

  CUtensorMap km, vm;
  const Plan plan = fp16 ? make_plan_fp16(head_dim, qpk, num_kv_heads) : make_plan(head_dim, qpk, num_kv_heads);
  const int fmt = fp16 ? 1 : (plan.r128 ? 2 : 0);
  if (!cached_kv_map(&km, fmt, k_data, head_dim, num_kv_heads, plan.hb, num_pages) ||
      !cached_kv_map(&vm, fmt, v_data, head_dim, num_kv_heads, plan.hb, num_pages)) {
    snprintf(iris::g_last_error, sizeof(iris::g_last_error), "cuTensorMapEncodeTiled failed (D=%d Hkv=%d pages=%lld)", head_dim,
             num_kv_heads, static_cast<long long>(num_pages));
    return IRIS_ECUDA;
  }

  DecodeParams p;
  p.query = static_cast<const __half*>(query);
  p.k_scale = static_cast<const uint8_t*>(k_scale);
  p.v_scale = static_cast<const uint8_t*>(v_scale);
  p.block_table = block_table;
  p.bt_stride = block_table_stride;
  p.seq_lens = seq_lens;
  p.out = output;
  p.out_lse = out_lse;
  p.rec_o = ws.rec_o;
  p.rec_lse = ws.rec_lse;
  p.prefix = ws.prefix;
  p.meta = ws.meta;
  p.err = error_word;
  p.num_pages = num_pages;
  p.batch = batch;
  p.hq = num_q_heads;
  p.hkv = num_kv_heads;
  p.max_pages = max_pages_per_seq;
  p.hb = 0;
  p.qpk = qpk;
  p.stages = 0;
  p.ranges = 0;
  p.combine_lanes = 1;
  p.out_mode = out_mode;
  p.scale_log2 = static_cast<float>(static_cast<double>(softmax_scale) * 1.4426950408889634);

  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  e = head_dim == 128 ? launch_decode<128>(plan, km, vm, p, device, s, max_ranges)
                      : launch_decode<64>(plan, km, vm, p, device, s, max_ranges);
  return e == cudaSuccess ? IRIS_OK : IRIS_ECUDA;
}


extern "C" int iris_b200_int4_paged_decode(const void* query, const void* k_data, const void* v_data,
                                           const void* k_scale, const void* v_scale, const int32_t* block_table,
                                           int64_t block_table_stride, const int32_t* seq_lens, void* output,
                                           float* out_lse, int32_t out_mode, int32_t batch, int32_t num_q_heads,
                                           int32_t num_kv_heads, int32_t head_dim, int64_t num_pages,
                                           int32_t page_size, int32_t max_pages_per_seq, float softmax_scale,
                                           void* workspace, size_t workspace_bytes, int32_t* error_word,
                                           void* stream) {
  return decode_entry(false, query, k_data, v_data, k_scale, v_scale, block_table, block_table_stride, seq_lens,
                      output, out_lse, out_mode, batch, num_q_heads, num_kv_heads, head_dim, num_pages, page_size,
                      max_pages_per_seq, softmax_scale, workspace, workspace_bytes, error_word, stream);
}

// The INT4 decode with its page ranges capped by the problem size (used by
// the allocation-free entry point, whose scratch is carved the same way).
int iris_decode_problem_sized(const void* query, const void* k_data, const void* v_data, const void* k_scale,
                              const void* v_scale, const int32_t* block_table, int64_t block_table_stride,
                              const int32_t* seq_lens, void* output, float* out_lse, int32_t out_mode, int32_t batch,
                              int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim, int64_t num_pages,
                              int32_t page_size, int32_t max_pages_per_seq, float softmax_scale, void* workspace,
                              size_t workspace_bytes, int32_t* error_word, void* stream) {
  return decode_entry(false, query, k_data, v_data, k_scale, v_scale, block_table, block_table_stride, seq_lens,
                      output, out_lse, out_mode, batch, num_q_heads, num_kv_heads, head_dim, num_pages, page_size,
                      max_pages_per_seq, softmax_scale, workspace, workspace_bytes, error_word, stream,
                      problem_ranges(batch, max_pages_per_seq));
}

extern "C" size_t iris_b200_fp16_decode_workspace_bytes(int32_t batch, int32_t num_q_heads, int32_t num_kv_heads,
                                                        int32_t head_dim, int32_t device) {
  if (batch <= 0 || num_q_heads <= 0 || num_kv_heads <= 0 || (head_dim != 64 && head_dim != 128)) return 0;
  if (num_q_heads % num_kv_heads != 0) return 0;
  return carve(nullptr, batch, num_q_heads, head_dim,
               max_ranges_for(num_q_heads / num_kv_heads, num_kv_heads, device_sms(device), true))
      .bytes;
}

extern "C" int iris_b200_fp16_paged_decode(const void* query, const void* k_cache, const void* v_cache,
                                           const int32_t* block_table, int64_t block_table_stride,
                                           const int32_t* seq_lens, void* output, float* out_lse, int32_t out_mode,
                                           int32_t batch, int32_t num_q_heads, int32_t num_kv_heads,
                                           int32_t head_dim, int64_t num_pages, int32_t page_size,
                                           int32_t max_pages_per_seq, float softmax_scale, void* workspace,
                                           size_t workspace_bytes, int32_t* error_word, void* stream) {
  return decode_entry(true, query, k_cache, v_cache, nullptr, nullptr, block_table, block_table_stride, seq_lens,
                      output, out_lse, out_mode, batch, num_q_heads, num_kv_heads, head_dim, num_pages, page_size,
                      max_pages_per_seq, softmax_scale, workspace, workspace_bytes, error_word, stream);
}

namespace {

int launch_merge(const float* parts_o, const float* parts_lse, int32_t num_parts, int64_t rows, int32_t head_dim,
                 int64_t o_stride, int64_t lse_stride, void* output, void* stream) {
  if (num_parts <= 0 || rows < 0 || head_dim <= 0 || parts_o == nullptr || parts_lse == nullptr || output == nullptr)
    return IRIS_EINVAL;
  if (rows == 0) return IRIS_OK;
  if (rows > 0x7fffffff) return IRIS_EUNSUPPORTED;
  clear_stale_cuda_error();
  merge_lse_kernel<<<static_cast<unsigned>(rows), 128, 0, static_cast<cudaStream_t>(stream)>>>(
      parts_o, parts_lse, num_parts, rows, head_dim, o_stride, lse_stride, static_cast<__half*>(output));
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    record_cuda_error(e, "merge_lse_kernel launch");
    return IRIS_ECUDA;
  }
  return IRIS_OK;
}

}  // namespace

extern "C" int iris_b200_merge_lse_partials(const float* parts_o, const float* parts_lse, int32_t num_parts,
                                            int64_t rows, int32_t head_dim, void* output, void* stream) {
  return launch_merge(parts_o, parts_lse, num_parts, rows, head_dim, rows * head_dim, rows, output, stream);
}

extern "C" int iris_b200_merge_lse_packed(const float* parts, int32_t num_parts, int64_t rows, int32_t head_dim,
                                          void* output, void* stream) {
  if (parts == nullptr) return IRIS_EINVAL;
  const int64_t part = rows * (head_dim + 1);
  return launch_merge(parts, parts + rows * head_dim, num_parts, rows, head_dim, part, part, output, stream);
}

extern "C" const char* iris_b200_last_cuda_error(void) { return iris::g_last_error; }

namespace {

// One thread waits, through the decode pipeline's bounded wait, on an
// mbarrier phase that nothing completes; after limit_ns it records the
// timeout bit and returns.  Exercises the failure path without a fault.
__global__ void bounded_wait_selftest_kernel(int32_t* err, uint64_t limit_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x != 0) return;
  iris::mbar_init(&bar, 1);
  iris::fence_barrier_init();
  iris::mbar_wait_bounded(iris::smem_u32(&bar), 0, err, limit_ns);  // phase 0 never completes
}

}  // namespace

extern "C" int iris_b200_selftest_bounded_wait(int32_t* error_word, int64_t limit_ns, void* stream) {
  if (error_word == nullptr || limit_ns <= 0 || limit_ns > 2000000000LL) return IRIS_EINVAL;
  iris::clear_stale_cuda_error();
  bounded_wait_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(error_word,
                                                                               static_cast<uint64_t>(limit_ns));
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    iris::record_cuda_error(e, "bounded_wait_selftest_kernel launch");
    return IRIS_ECUDA;
  }
  return IRIS_OK;
}

extern "C" int iris_b200_version(void) { return 100; }

extern "C" const char* iris_b200_status_string(int status) {
  switch (status) {
    case IRIS_OK: return "ok";
    case IRIS_EINVAL: return "invalid argument";
    case IRIS_EUNSUPPORTED: return "unsupported shape";
    case IRIS_EALIGN: return "pointer not aligned as required";
    case IRIS_ECUDA: return "CUDA runtime error";
    case IRIS_EWORKSPACE: return "workspace too small";
    default: return "unknown status";
  }
}
