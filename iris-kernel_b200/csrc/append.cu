// Fused RoPE(K) + group-32 symmetric INT4 quantisation + low-nibble-first
// packing + paged append, for sm_100a.
//
// Replaces the reference kernel _rope_int4_paged_append
// (src/iris_kernel/fused_kv.py:419-597) and reproduces, bit for bit, the
// eager semantics of torch_eager_append (src/iris_kernel/torch_eager_kv.py:
// 110-337): RoPE with an fp16 rounding after every op (:38-47), fp32 group
// absmax, scale = fp16(max(amax / 7, 2^-14)) with an IEEE division (:69-81),
// q = clamp(rint(x / scale), -7, 7) with an IEEE division and
// round-half-to-even (:83-86), byte = q[2i] & 0xF | (q[2i+1] & 0xF) << 4
// (:104-107).
//
// Layout of the work: one thread owns one 32-dim quantisation group of one
// (token, kv-head) row, for both K and V (D/32 threads per row), so the group
// absmax and scale need no communication and the 16 packed bytes leave in
// one vector store.  The kernel is HBM-bound: per (token, head) it moves 4D
// bytes in and D + D/8 bytes out.  Small batches (decode steps) use a
// latency-shaped form instead: one thread per half group, two adjacent lanes
// sharing the absmax, in CTAs small enough to run beside a decode kernel.
#include <cstdlib>
#include <map>
#include <mutex>
#include <utility>

#include "common.cuh"

namespace iris {

// Division of non-negative 32-bit integers n < 2^31 by a divisor fixed at
// launch: q = (umulhi(n, m) + n) >> l with l = ceil(log2 d) and
// m = floor(2^32 (2^l - d) / d) + 1 (Granlund & Montgomery, "Division by
// Invariant Integers using Multiplication", 1994).
struct FastDiv {
  uint32_t d, m, l;
  static FastDiv make(uint32_t d) {
    FastDiv f;
    f.d = d;
    f.l = 0;
    while ((1ull << f.l) < d) ++f.l;
    f.m = static_cast<uint32_t>(((1ull << 32) * ((1ull << f.l) - d)) / d + 1);
    return f;
  }
  IRIS_DEV uint32_t div(uint32_t n) const { return (__umulhi(n, m) + n) >> l; }
};

struct AppendParams {
  const __half* key;
  const __half* value;
  const int32_t* positions;
  const int32_t* slots;
  const __half* cos_cache;
  const __half* sin_cache;
  uint8_t* k_data;
  uint8_t* v_data;
  __half* k_scale;
  __half* v_scale;
  int64_t num_tokens;
  int64_t max_position;
  int64_t num_slots;  // num_pages * page_size
  int32_t num_heads;
  int32_t page_size;
  FastDiv heads_div;  // row -> (token, head)
  FastDiv page_div;   // slot -> (page, offset)
  int32_t* err;
  int64_t prefetch_rows;  // one-pass kernel: L2 prefetch distance in rows (0: none)
};

// Batches of at most this many tokens are validated inside the append kernel
// (ranges and duplicate slots, by every CTA), with no check kernel before it.
constexpr int64_t kInlineCheckTokens = IRIS_APPEND_INLINE_CHECK_TOKENS;

// 32-byte read-only load (sm_100 vector width), 32-byte aligned address.
IRIS_DEV void ldg_nc_v8(const void* p, uint4& a, uint4& b) {
  asm volatile("ld.global.nc.v8.u32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(a.x), "=r"(a.y), "=r"(a.z), "=r"(a.w), "=r"(b.x), "=r"(b.y), "=r"(b.z), "=r"(b.w)
               : "l"(p));
}

IRIS_DEV uint4 ldg_nc_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}


// fp16 group scale from the group's absmax, exactly as the eager reference.
//
// amax / 7 is rounded with one Markstein residual step instead of a division:
// amax = A 2^e with an 11-bit A, so amax / 7 either is exact (7 | A) or has a
// non-terminating period-3 binary expansion that stays at least ~2^-28
// (relative) away from every fp32 rounding midpoint, while the corrected
// estimate is within 2^-43 before its final rounding: both round alike.
// Checked against the IEEE division for all 31,744 finite fp16 values.
IRIS_DEV __half group_scale(__half amax) {
  const float a = __half2float(amax);
  float s;
  if (a <= 65504.0f) {
    const float r7 = 0.142857149f;  // fp32(1/7)
    const float y = __fmul_rn(a, r7);
    s = fmaf(fmaf(-y, 7.0f, a), r7, y);
  } else {
    s = __fdiv_rn(a, 7.0f);  // Inf / NaN
  }
  const float tiny = 6.103515625e-05f;  // 2^-14 = torch.finfo(float16).tiny
  s = (s < tiny) ? tiny : s;            // NaN stays NaN (torch clamp_min)
  return __float2half_rn(s);
}

// Reference semantics, IEEE division: q = clamp(rint(x / scale), -7, 7).
// Used for non-finite scales (a group holding Inf or NaN).
IRIS_DEV uint32_t quant_pack8_ieee(const __half2 (&v)[4], float scale) {
  uint32_t word = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(v[i]);
    int q0 = __float2int_rn(__fdiv_rn(f.x, scale));
    int q1 = __float2int_rn(__fdiv_rn(f.y, scale));
    q0 = min(7, max(-7, q0));
    q1 = min(7, max(-7, q1));
    word |= (static_cast<uint32_t>(q0) & 0xFu) << (8 * i);
    word |= (static_cast<uint32_t>(q1) & 0xFu) << (8 * i + 4);
  }
  return word;
}

IRIS_DEV float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}


// The same result without a division, for a finite group scale.
//
// x and scale are fp16 values, so x / scale = X 2^a / (S 2^b) with 11-bit
// integers X, S.  If the quotient is not exactly a half-integer it is at
// least 2^-13 away from one (for |q| >= 1/4 the numerator x - (k+1/2) scale
// is a non-zero multiple of 2^(e_scale - 12) and scale < 2^(e_scale + 1)),
// while the fp32 quotient is off by at most 7.5 * 2^-24: IEEE rounding and
// round-half-even then agree with any estimate that close.  y = x * rcp(scale) is within ~2^-21 relative;
// one Markstein residual step (Markstein 1990: e = x - y*scale, exact in one
// FMA since it has at most 13 significant bits; y += e * rcp) lands within
// |q| 2^-43 of q before rounding, so exact half-integers come out exact, so the ties
// also round to even.  Adding 2^23 + 16 rounds y to the nearest integer,
// ties to even, and leaves (q + 16) mod 16 -- the two's-complement nibble --
// in the low four mantissa bits.  |x| <= amax and scale = fp16(amax / 7)
// (or 2^-14) keep |q| <= 7, so the reference's clamp never binds here.
// Checked against the IEEE path on every exact tie and a dense sweep
// (tests/test_gpu_append.py).
//
// 8 fp16 values (one 16-byte vector) -> 8 nibbles (one 32-bit word), for a
// finite scale.
IRIS_DEV uint32_t quant_pack_vec(const uint4& raw, float scale, float r) {
  const __half2* v = reinterpret_cast<const __half2*>(&raw);
  // the same operations on value pairs with the sm_100 packed fp32 forms
  // (each lane rounds as its scalar counterpart does)
  const float kRound = 8388624.0f;  // 2^23 + 16
  const float2 r2 = make_float2(r, r), ns2 = make_float2(-scale, -scale), k2 = make_float2(kRound, kRound);
  uint32_t b[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(v[i]);
    float2 y = __fmul2_rn(f, r2);
    y = __ffma2_rn(__ffma2_rn(y, ns2, f), r2, y);  // y + (f - y*scale) * r
    const float2 z = __fadd2_rn(y, k2);
    b[2 * i] = __float_as_uint(z.x);
    b[2 * i + 1] = __float_as_uint(z.y);
  }
  // byte i of the word = nibble(2i) | nibble(2i+1) << 4: gather the low bytes
  // of the even and of the odd values, then merge the nibbles
  const uint32_t ev = __byte_perm(__byte_perm(b[0], b[2], 0x0040), __byte_perm(b[4], b[6], 0x0040), 0x5410);
  const uint32_t od = __byte_perm(__byte_perm(b[1], b[3], 0x0040), __byte_perm(b[5], b[7], 0x0040), 0x5410);
  return (ev & 0x0F0F0F0Fu) | ((od << 4) & 0xF0F0F0F0u);
}

IRIS_DEV __half2 habs_max_vec(const uint4& raw) {
  const __half2* v = reinterpret_cast<const __half2*>(&raw);
  return __hmax2_nan(__hmax2_nan(__habs2(v[0]), __habs2(v[1])), __hmax2_nan(__habs2(v[2]), __habs2(v[3])));
}

// One 32-dim quantisation group (4 vectors): fp16 scale and 4 packed words.
IRIS_DEV void quant_group(const uint4 (&g)[4], __half& scale16, uint4& packed) {
  __half2 m = __hmax2_nan(__hmax2_nan(habs_max_vec(g[0]), habs_max_vec(g[1])),
                          __hmax2_nan(habs_max_vec(g[2]), habs_max_vec(g[3])));
  scale16 = group_scale(__hmax_nan(__low2half(m), __high2half(m)));
  const float sc = __half2float(scale16);
  if (fabsf(sc) <= 3.0e38f) {  // finite: division-free path (one branch per group)
    const float r = rcp_approx(sc);
    packed.x = quant_pack_vec(g[0], sc, r);
    packed.y = quant_pack_vec(g[1], sc, r);
    packed.z = quant_pack_vec(g[2], sc, r);
    packed.w = quant_pack_vec(g[3], sc, r);
  } else {
    const __half2* v = reinterpret_cast<const __half2*>(g);
    const __half2 v0[4] = {v[0], v[1], v[2], v[3]}, v1[4] = {v[4], v[5], v[6], v[7]};
    const __half2 v2[4] = {v[8], v[9], v[10], v[11]}, v3[4] = {v[12], v[13], v[14], v[15]};
    packed.x = quant_pack8_ieee(v0, sc);
    packed.y = quant_pack8_ieee(v1, sc);
    packed.z = quant_pack8_ieee(v2, sc);
    packed.w = quant_pack8_ieee(v3, sc);
  }
}

// One thread owns one 32-dim quantisation group of one (token, kv-head) row,
// for both K and V: D/32 threads per row.  The group's absmax and scale are
// thread-local, its 16 packed bytes leave in one vector store.  The RoPE
// partner group (dims +-D/2) is read again by this thread (an L1 hit: the
// partner thread loads it too).
template <int D>
struct AppendCfg {
  static constexpr int kTpr = D / 32;                    // threads per row
  static constexpr int kHalf = kTpr / 2;                 // partner distance in groups
  static constexpr int kRows = 128 / kTpr;               // rows per CTA
  static constexpr int kThreads = kRows * kTpr;
};

constexpr int32_t kRejectBits = IRIS_ERR_SLOT_RANGE | IRIS_ERR_POS_NEGATIVE | IRIS_ERR_POS_RANGE | IRIS_ERR_DUP_SLOT;

// Validation of a small batch (at most kInlineCheckTokens tokens) inside an
// append kernel, done by every CTA as append_check_kernel does it for a large
// one: ranges, then each live slot counted against all slots (16-byte
// broadcast reads of a shared copy).  Every thread of the CTA calls it; it
// returns whether the batch is rejected, and CTA 0 records the bits.
template <int kThreads>
IRIS_DEV bool inline_batch_check(const int32_t* __restrict__ slots, const int32_t* __restrict__ positions, int T,
                                 int64_t num_slots, int64_t max_position, int32_t* err) {
  __shared__ __align__(16) int32_t s_slot[kInlineCheckTokens];
  const int tid = threadIdx.x;
  const int T4 = (T + 3) & ~3;
  int32_t bits = 0;
  for (int i = tid; i < T4; i += kThreads) {
    int32_t s = -1;
    if (i < T) {
      s = __ldg(slots + i);
      if (s >= 0) {
        const int32_t ps = __ldg(positions + i);
        if (static_cast<int64_t>(s) >= num_slots) bits |= IRIS_ERR_SLOT_RANGE;
        if (ps < 0) bits |= IRIS_ERR_POS_NEGATIVE;
        else if (static_cast<int64_t>(ps) >= max_position) bits |= IRIS_ERR_POS_RANGE;
      }
    }
    s_slot[i] = s;
  }
  __syncthreads();
  for (int i = tid; i < T; i += kThreads) {
    const int32_t s = s_slot[i];
    if (s < 0 || static_cast<int64_t>(s) >= num_slots) continue;
    int hits = 0;
    for (int j = 0; j < T4; j += 4) {
      const int4 v = *reinterpret_cast<const int4*>(s_slot + j);
      hits += (v.x == s) + (v.y == s) + (v.z == s) + (v.w == s);
    }
    if (hits > 1) bits |= IRIS_ERR_DUP_SLOT;
  }
  if (blockIdx.x == 0 && bits) set_error(err, bits);
  return __syncthreads_or(bits != 0);
}

// kWide: the group's 64 bytes (and its cos / sin rows) arrive in two 32-byte
// loads, so every sector a warp's load touches is used whole (with 16-byte
// loads the lanes' 64-byte stride fetches each sector twice and the L1
// throughput bounds the kernel).  Needs 32-byte aligned key / value / cos /
// sin bases.
template <int D, bool kWide>
__global__ void __launch_bounds__(AppendCfg<D>::kThreads) rope_int4_append_kernel(const AppendParams p) {
  using C = AppendCfg<D>;
  const int tid = threadIdx.x;
  const int c = tid % C::kTpr;  // group within the row
  const uint32_t row = blockIdx.x * C::kRows + tid / C::kTpr;
  const uint32_t nrows = static_cast<uint32_t>(p.num_tokens) * static_cast<uint32_t>(p.num_heads);
  const bool in_range = row < nrows;
  const uint32_t rr = in_range ? row : 0u;  // rows past the end read row 0 and store nothing
  const uint32_t tok = p.heads_div.div(rr);
  const uint32_t h = rr - tok * static_cast<uint32_t>(p.num_heads);
  const int32_t slot = __ldg(p.slots + tok);
  const int32_t pos = __ldg(p.positions + tok);

  const bool lo_half = c < C::kHalf;
  const int pair = lo_half ? c : c - C::kHalf;  // group index into cos/sin
  const int partner = lo_half ? c + C::kHalf : c - C::kHalf;
  const __half* krow = p.key + static_cast<size_t>(rr) * D;
  const __half* vrow = p.value + static_cast<size_t>(rr) * D;
  uint4 ko[4], kp[4], vo[4], cs[4], sn[4];
  // K / V loads of one group (they depend on neither the slot nor the position)
  const auto load_kv = [&](int i) {
    if constexpr (kWide) {
      ldg_nc_v8(krow + 32 * c + 8 * i, ko[i], ko[i + 1]);
      ldg_nc_v8(krow + 32 * partner + 8 * i, kp[i], kp[i + 1]);
      ldg_nc_v8(vrow + 32 * c + 8 * i, vo[i], vo[i + 1]);
    } else {
      ko[i] = ldg_nc_v4(krow + 32 * c + 8 * i);
      kp[i] = ldg_nc_v4(krow + 32 * partner + 8 * i);
      vo[i] = ldg_nc_v4(vrow + 32 * c + 8 * i);
    }
  };
  constexpr int kStep = kWide ? 2 : 1;  // 16-byte vectors per load
  if (tid == 0 && p.prefetch_rows > 0) {
    // the K / V rows of the CTA about one resident wave later go to L2 now,
    // so DRAM keeps streaming while this wave computes
    const int64_t r0 = static_cast<int64_t>(blockIdx.x) * C::kRows + p.prefetch_rows;
    if (r0 < nrows) {
      const int64_t n = nrows - r0 < C::kRows ? nrows - r0 : C::kRows;
      prefetch_l2_bulk(p.key + r0 * D, static_cast<uint32_t>(n * D * 2));
      prefetch_l2_bulk(p.value + r0 * D, static_cast<uint32_t>(n * D * 2));
    }
  }
  if (!in_range || slot < 0) return;  // no collective operations below
  {
    int32_t bits = 0;
    if (static_cast<int64_t>(slot) >= p.num_slots) bits |= IRIS_ERR_SLOT_RANGE;
    if (pos < 0) bits |= IRIS_ERR_POS_NEGATIVE;
    else if (static_cast<int64_t>(pos) >= p.max_position) bits |= IRIS_ERR_POS_RANGE;
    if (bits) {  // never touch memory outside the cache / RoPE tables
      if (h == 0 && c == 0) set_error(p.err, bits);
      return;
    }
  }
  const __half* crow = p.cos_cache + static_cast<size_t>(pos) * (D / 2) + 32 * pair;
  const __half* srow = p.sin_cache + static_cast<size_t>(pos) * (D / 2) + 32 * pair;
#pragma unroll
  for (int i = 0; i < 4; i += kStep) {
    load_kv(i);
    if constexpr (kWide) {
      ldg_nc_v8(crow + 8 * i, cs[i], cs[i + 1]);
      ldg_nc_v8(srow + 8 * i, sn[i], sn[i + 1]);
    } else {
      cs[i] = ldg_nc_v4(crow + 8 * i);
      sn[i] = ldg_nc_v4(srow + 8 * i);
    }
  }

  // ---- RoPE, fp16 rounding after each op ----
  // low half:  y = x1*cos - x2*sin   (own = x1, partner = x2)
  // high half: y = x2*cos + x1*sin   (own = x2, partner = x1)
  // written as own*cos + (+-partner)*sin; negation is exact.
  uint4 kr[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __half2* own = reinterpret_cast<const __half2*>(&ko[i]);
    const __half2* par = reinterpret_cast<const __half2*>(&kp[i]);
    const __half2* cc = reinterpret_cast<const __half2*>(&cs[i]);
    const __half2* ss = reinterpret_cast<const __half2*>(&sn[i]);
    __half2* out = reinterpret_cast<__half2*>(&kr[i]);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const __half2 pj = lo_half ? __hneg2(par[j]) : par[j];
      out[j] = __hadd2(__hmul2_rn(own[j], cc[j]), __hmul2_rn(pj, ss[j]));
    }
  }

  // ---- quantise, pack, store ----
  __half ks, vs;
  uint4 kw, vw;
  quant_group(kr, ks, kw);
  quant_group(vo, vs, vw);
  // Everything above overlaps the check kernel (programmatic launch); the
  // stores wait for it.  A slot / position / duplicate error it recorded
  // means the batch is rejected: nothing is written, as the reference raises
  // before it writes.
  grid_dependency_wait();
  if (p.err != nullptr && (*p.err & kRejectBits) != 0) return;
  const uint32_t page = p.page_div.div(static_cast<uint32_t>(slot));
  const uint32_t off = static_cast<uint32_t>(slot) - page * static_cast<uint32_t>(p.page_size);
  const size_t crow_idx = (static_cast<size_t>(page) * p.page_size + off) * p.num_heads + h;  // cache row
  *reinterpret_cast<uint4*>(p.k_data + crow_idx * (D / 2) + 16 * c) = kw;
  *reinterpret_cast<uint4*>(p.v_data + crow_idx * (D / 2) + 16 * c) = vw;
  p.k_scale[crow_idx * (D / 32) + c] = ks;
  p.v_scale[crow_idx * (D / 32) + c] = vs;
}

// A small batch (at most kInlineCheckTokens tokens): one thread per half
// quantisation group (16 dims), so a thread holds half the loads of the
// kernel above in flight, and 64-thread CTAs of at most 64 registers a thread
// (4096 registers, what a decode kernel at 3 CTAs of 160 threads x 128
// registers leaves free on an SM: the append of a decode step runs on the
// SMs beside the decode).  Every CTA validates the whole batch before storing
// (no check kernel before the launch); the K / V loads are issued first and
// overlap that check.  A group's two halves are adjacent lanes and share
// their absmax with one shuffle, so the scale and the packed bytes are those
// of the one-thread-per-group kernel.
template <int D>
struct SmallAppendCfg {
  static constexpr int kTpr = D / 16;         // threads per row: half groups
  static constexpr int kHalf = kTpr / 2;      // partner distance (D/2 dims) in half groups
  static constexpr int kRows = 64 / kTpr;     // rows per CTA
  static constexpr int kThreads = kRows * kTpr;
};

template <int D, bool kWide>
__global__ void __launch_bounds__(SmallAppendCfg<D>::kThreads, 16) rope_int4_append_small_kernel(const AppendParams p) {
  using C = SmallAppendCfg<D>;
  const int tid = threadIdx.x;
  const int c = tid % C::kTpr;  // half group within the row
  const int g = c >> 1, hf = c & 1;
  const uint32_t row = blockIdx.x * C::kRows + tid / C::kTpr;
  const uint32_t nrows = static_cast<uint32_t>(p.num_tokens) * static_cast<uint32_t>(p.num_heads);
  const bool in_range = row < nrows;
  const uint32_t rr = in_range ? row : 0u;  // rows past the end read row 0 and store nothing
  const uint32_t tok = p.heads_div.div(rr);
  const uint32_t h = rr - tok * static_cast<uint32_t>(p.num_heads);
  const int32_t slot = __ldg(p.slots + tok);
  const int32_t pos = __ldg(p.positions + tok);

  const bool lo_half = c < C::kHalf;
  const int pair = lo_half ? c : c - C::kHalf;  // half group index into cos/sin
  const int partner = lo_half ? c + C::kHalf : c - C::kHalf;
  const __half* krow = p.key + static_cast<size_t>(rr) * D;
  const __half* vrow = p.value + static_cast<size_t>(rr) * D;
  uint4 ko[2], kp[2], vo[2], cs[2], sn[2];
  if constexpr (kWide) {
    ldg_nc_v8(krow + 16 * c, ko[0], ko[1]);
    ldg_nc_v8(krow + 16 * partner, kp[0], kp[1]);
    ldg_nc_v8(vrow + 16 * c, vo[0], vo[1]);
  } else {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      ko[i] = ldg_nc_v4(krow + 16 * c + 8 * i);
      kp[i] = ldg_nc_v4(krow + 16 * partner + 8 * i);
      vo[i] = ldg_nc_v4(vrow + 16 * c + 8 * i);
    }
  }
  const bool batch_bad = inline_batch_check<C::kThreads>(p.slots, p.positions, static_cast<int>(p.num_tokens),
                                                         p.num_slots, p.max_position, p.err);
  // from here on a row's threads leave together (the pair shuffle below needs both halves)
  if (batch_bad || !in_range || slot < 0) return;
  {
    int32_t bits = 0;
    if (static_cast<int64_t>(slot) >= p.num_slots) bits |= IRIS_ERR_SLOT_RANGE;
    if (pos < 0) bits |= IRIS_ERR_POS_NEGATIVE;
    else if (static_cast<int64_t>(pos) >= p.max_position) bits |= IRIS_ERR_POS_RANGE;
    if (bits) return;  // recorded by the batch check; never touch memory outside the tables
  }
  const __half* crow = p.cos_cache + static_cast<size_t>(pos) * (D / 2) + 16 * pair;
  const __half* srow = p.sin_cache + static_cast<size_t>(pos) * (D / 2) + 16 * pair;
  if constexpr (kWide) {
    ldg_nc_v8(crow, cs[0], cs[1]);
    ldg_nc_v8(srow, sn[0], sn[1]);
  } else {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      cs[i] = ldg_nc_v4(crow + 8 * i);
      sn[i] = ldg_nc_v4(srow + 8 * i);
    }
  }

  // RoPE with fp16 rounding after each op, as in the kernel above
  uint4 kr[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const __half2* own = reinterpret_cast<const __half2*>(&ko[i]);
    const __half2* par = reinterpret_cast<const __half2*>(&kp[i]);
    const __half2* cc = reinterpret_cast<const __half2*>(&cs[i]);
    const __half2* ss = reinterpret_cast<const __half2*>(&sn[i]);
    __half2* out = reinterpret_cast<__half2*>(&kr[i]);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const __half2 pj = lo_half ? __hneg2(par[j]) : par[j];
      out[j] = __hadd2(__hmul2_rn(own[j], cc[j]), __hmul2_rn(pj, ss[j]));
    }
  }

  // the group's absmax over both halves (the max is exact and order-free)
  const unsigned pair_mask = 3u << ((threadIdx.x & 31) & ~1);
  const auto group_absmax = [&](const uint4 (&v)[2]) {
    const __half2 m = __hmax2_nan(habs_max_vec(v[0]), habs_max_vec(v[1]));
    const __half mine = __hmax_nan(__low2half(m), __high2half(m));
    const unsigned short other = __shfl_xor_sync(pair_mask, __half_as_ushort(mine), 1);
    return __hmax_nan(mine, __ushort_as_half(other));
  };
  const auto quant_half = [&](const uint4 (&v)[2], __half& scale16, uint2& packed) {
    scale16 = group_scale(group_absmax(v));
    const float sc = __half2float(scale16);
    if (fabsf(sc) <= 3.0e38f) {
      const float r = rcp_approx(sc);
      packed.x = quant_pack_vec(v[0], sc, r);
      packed.y = quant_pack_vec(v[1], sc, r);
    } else {
      const __half2* x = reinterpret_cast<const __half2*>(v);
      const __half2 x0[4] = {x[0], x[1], x[2], x[3]}, x1[4] = {x[4], x[5], x[6], x[7]};
      packed.x = quant_pack8_ieee(x0, sc);
      packed.y = quant_pack8_ieee(x1, sc);
    }
  };
  __half ks, vs;
  uint2 kw, vw;
  quant_half(kr, ks, kw);
  quant_half(vo, vs, vw);
  // an earlier rejected batch whose error is still pending refuses this one too
  if (p.err != nullptr && (*p.err & kRejectBits) != 0) return;
  const uint32_t page = p.page_div.div(static_cast<uint32_t>(slot));
  const uint32_t off = static_cast<uint32_t>(slot) - page * static_cast<uint32_t>(p.page_size);
  const size_t crow_idx = (static_cast<size_t>(page) * p.page_size + off) * p.num_heads + h;  // cache row
  *reinterpret_cast<uint2*>(p.k_data + crow_idx * (D / 2) + 16 * g + 8 * hf) = kw;
  *reinterpret_cast<uint2*>(p.v_data + crow_idx * (D / 2) + 16 * g + 8 * hf) = vw;
  if (hf == 0) {
    p.k_scale[crow_idx * (D / 32) + g] = ks;
    p.v_scale[crow_idx * (D / 32) + g] = vs;
  }
}

// One thread per token: range checks and duplicate detection through a
// slot bitmap (one bit per cache slot, cleared by the caller-side memset).
__global__ void append_check_kernel(const int32_t* __restrict__ positions, const int32_t* __restrict__ slots,
                                    int64_t num_tokens, int64_t max_position, int64_t num_slots,
                                    uint32_t* __restrict__ bitmap, int32_t* err) {
  grid_dependents_launch();  // the append kernel may start loading meanwhile
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= num_tokens) return;
  const int32_t s = slots[i];
  if (s < 0) return;
  int32_t bits = 0;
  if (static_cast<int64_t>(s) >= num_slots) {
    bits |= IRIS_ERR_SLOT_RANGE;
  } else {
    const uint32_t bit = 1u << (s & 31);
    if (atomicOr(bitmap + (s >> 5), bit) & bit) bits |= IRIS_ERR_DUP_SLOT;
  }
  const int32_t pos = positions[i];
  if (pos < 0) bits |= IRIS_ERR_POS_NEGATIVE;
  else if (static_cast<int64_t>(pos) >= max_position) bits |= IRIS_ERR_POS_RANGE;
  if (bits) set_error(err, bits);
}

// Standalone group-32 INT4 quantise + pack of a contiguous [rows, D] fp16
// tensor (rows = T * H): the append's quantiser without RoPE or paging.  One
// thread per 32-value group: 64 bytes in, 16 packed bytes + one fp16 scale
// out.
__global__ void __launch_bounds__(256) quantize_pack_kernel(const __half* __restrict__ x, uint8_t* __restrict__ packed,
                                                            __half* __restrict__ scales, int64_t groups) {
  const int64_t g = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (g >= groups) return;
  const __half* src = x + g * 32;
  uint4 v[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = ldg_nc_v4(src + 8 * i);
  __half sc;
  uint4 w;
  quant_group(v, sc, w);
  *reinterpret_cast<uint4*>(packed + g * 16) = w;
  scales[g] = sc;
}

// FP16 paged append (the reference's fused_rope_fp16_append): RoPE over the
// first rotary_dim dims of K with fp16 rounding after every operation, the
// rest of K and all of V copied, into k_cache / v_cache [pages, 16, H, D]
// fp16 (row of (slot, head) at (slot * H + head) * D).  VEC: one thread per
// 8-dim chunk (D % 8 == 0, rotary_dim % 16 == 0); otherwise one per dim.
struct Fp16AppendParams {
  const __half* key;
  const __half* value;
  const int32_t* positions;
  const int32_t* slots;
  const __half* cos_cache;
  const __half* sin_cache;
  __half* k_cache;
  __half* v_cache;
  int64_t num_tokens;
  int64_t max_position;
  int64_t num_slots;
  int32_t num_heads, head_dim, rotary_dim;
  int32_t* err;
  FastDiv row_div;   // thread -> (row, chunk): by threads per row
  FastDiv head_div;  // row -> (token, head)
};

// W: dims per thread (16: 32-byte loads, 8: 16-byte loads, 1: scalar).
// k32: the launch has fewer than 2^31 threads, so a thread's row, token and
// head come from 32-bit multiply-shift divisions instead of 64-bit ones.
template <int W, bool kInline, bool k32>
__global__ void __launch_bounds__(256) rope_fp16_append_kernel(const Fp16AppendParams p) {
  constexpr bool VEC = W >= 8;
  constexpr int NV = W / 8;  // 16-byte vectors per thread and tensor
  const int per_row = p.head_dim / W;
  int64_t row, tok, h;
  int c;
  if constexpr (k32) {
    const uint32_t idx = blockIdx.x * blockDim.x + threadIdx.x;
    const uint32_t r32 = p.row_div.div(idx);
    const uint32_t t32 = p.head_div.div(r32);
    row = r32;
    c = static_cast<int>(idx - r32 * static_cast<uint32_t>(per_row));
    tok = t32;
    h = r32 - t32 * static_cast<uint32_t>(p.num_heads);
  } else {
    const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    row = idx / per_row;
    c = static_cast<int>(idx - row * per_row);
    tok = row / p.num_heads;
    h = row - tok * p.num_heads;
  }
  bool batch_bad = false;
  if constexpr (kInline)  // a small batch: every CTA validates it (no check kernel before the launch)
    batch_bad = inline_batch_check<256>(p.slots, p.positions, static_cast<int>(p.num_tokens), p.num_slots,
                                        p.max_position, p.err);
  if (row >= p.num_tokens * p.num_heads) return;
  const int32_t slot = __ldg(p.slots + tok);
  if (slot < 0) return;
  const int32_t pos = __ldg(p.positions + tok);
  {
    int32_t bits = 0;
    if (static_cast<int64_t>(slot) >= p.num_slots) bits |= IRIS_ERR_SLOT_RANGE;
    if (pos < 0) bits |= IRIS_ERR_POS_NEGATIVE;
    else if (static_cast<int64_t>(pos) >= p.max_position) bits |= IRIS_ERR_POS_RANGE;
    if (bits) {
      if (h == 0 && c == 0) set_error(p.err, bits);
      return;
    }
  }
  const int d0 = c * W;
  const int half = p.rotary_dim / 2;
  const __half* krow = p.key + row * p.head_dim;
  const __half* vrow = p.value + row * p.head_dim;
  const int64_t dst = (static_cast<int64_t>(slot) * p.num_heads + h) * p.head_dim + d0;
  if constexpr (VEC) {
    const auto load = [](const __half* src, uint4 (&dst)[NV]) {
      if constexpr (NV == 2)
        ldg_nc_v8(src, dst[0], dst[1]);
      else
        dst[0] = ldg_nc_v4(src);
    };
    uint4 k[NV], v[NV];
    load(krow + d0, k);
    load(vrow + d0, v);
    if (d0 < p.rotary_dim) {
      const bool lo = d0 < half;
      const int j = lo ? d0 : d0 - half;  // cos/sin column
      uint4 par[NV], cs[NV], sn[NV];
      load(krow + (lo ? d0 + half : d0 - half), par);
      load(p.cos_cache + static_cast<int64_t>(pos) * half + j, cs);
      load(p.sin_cache + static_cast<int64_t>(pos) * half + j, sn);
#pragma unroll
      for (int q = 0; q < NV; ++q) {
        __half2* own = reinterpret_cast<__half2*>(&k[q]);
        const __half2* pr = reinterpret_cast<const __half2*>(&par[q]);
        const __half2* cc = reinterpret_cast<const __half2*>(&cs[q]);
        const __half2* ss = reinterpret_cast<const __half2*>(&sn[q]);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const __half2 pi = lo ? __hneg2(pr[i]) : pr[i];
          own[i] = __hadd2(__hmul2_rn(own[i], cc[i]), __hmul2_rn(pi, ss[i]));
        }
      }
    }
    grid_dependency_wait();  // the check kernel before this launch has finished
    if (batch_bad || (p.err != nullptr && (*p.err & kRejectBits) != 0)) return;
#pragma unroll
    for (int q = 0; q < NV; ++q) {
      *reinterpret_cast<uint4*>(p.k_cache + dst + 8 * q) = k[q];
      *reinterpret_cast<uint4*>(p.v_cache + dst + 8 * q) = v[q];
    }
  } else {
    __half k = krow[d0];
    const __half v = vrow[d0];
    if (d0 < p.rotary_dim) {
      const bool lo = d0 < half;
      const int j = lo ? d0 : d0 - half;
      const __half par = krow[lo ? d0 + half : d0 - half];
      const __half cs = p.cos_cache[static_cast<int64_t>(pos) * half + j];
      const __half sn = p.sin_cache[static_cast<int64_t>(pos) * half + j];
      k = __hadd(__hmul_rn(k, cs), __hmul_rn(lo ? __hneg(par) : par, sn));
    }
    grid_dependency_wait();
    if (batch_bad || (p.err != nullptr && (*p.err & kRejectBits) != 0)) return;
    p.k_cache[dst] = k;
    p.v_cache[dst] = v;
  }
}

template <int W>
static cudaError_t launch_fp16_append(const cudaLaunchConfig_t& cfg, const Fp16AppendParams& p, bool small,
                                      bool k32) {
  return k32 ? (small ? cudaLaunchKernelEx(&cfg, rope_fp16_append_kernel<W, true, true>, p)
                      : cudaLaunchKernelEx(&cfg, rope_fp16_append_kernel<W, false, true>, p))
             : (small ? cudaLaunchKernelEx(&cfg, rope_fp16_append_kernel<W, true, false>, p)
                      : cudaLaunchKernelEx(&cfg, rope_fp16_append_kernel<W, false, false>, p));
}

// L2 prefetch distance of the one-pass kernel in quarters of a resident wave
// (IRIS_APPEND_PREFETCH=<quarters> overrides it, 0 turns it off; tuning).
static int append_prefetch_quarters() {
  static const int quarters = [] {
    const char* e = getenv("IRIS_APPEND_PREFETCH");
    return e != nullptr ? atoi(e) : 2;
  }();
  return quarters;
}

// IRIS_APPEND_WIDE=0 keeps the one-pass kernel on 16-byte loads (tuning).
static bool append_wide_enabled() {
  static const bool on = [] {
    const char* e = getenv("IRIS_APPEND_WIDE");
    return !(e != nullptr && e[0] == '0');
  }();
  return on;
}

// Resident CTAs per SM x SMs of a kernel, queried once per (kernel, device).
static cudaError_t resident_ctas(const void* fn, int threads, int smem, int64_t* out) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, int64_t> cache;
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(mu);
  const auto key = std::make_pair(fn, device);
  auto it = cache.find(key);
  if (it == cache.end()) {
    int n_sm = 0, n_occ = 0;
    e = cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, device);
    if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n_occ, fn, threads, smem);
    if (e != cudaSuccess) return e;
    it = cache.emplace(key, static_cast<int64_t>(n_sm) * n_occ).first;
  }
  *out = it->second;
  return cudaSuccess;
}

template <int D>
static cudaError_t launch_append(const AppendParams& p, cudaStream_t stream) {
  const int64_t rows = p.num_tokens * p.num_heads;
  if (rows == 0) return cudaSuccess;
  const auto aligned32 = [](const void* a) { return (reinterpret_cast<uintptr_t>(a) & 31) == 0; };
  const bool wide = aligned32(p.key) && aligned32(p.value) && aligned32(p.cos_cache) && aligned32(p.sin_cache) &&
                    append_wide_enabled();
  AppendParams q = p;
  q.prefetch_rows = 0;
  if (p.num_tokens <= kInlineCheckTokens) {  // a small batch checks itself; an ordinary launch
    using S = SmallAppendCfg<D>;
    const auto fn = wide ? rope_int4_append_small_kernel<D, true> : rope_int4_append_small_kernel<D, false>;
    fn<<<static_cast<unsigned>((rows + S::kRows - 1) / S::kRows), S::kThreads, 0, stream>>>(q);
    return cudaGetLastError();
  }
  using C = AppendCfg<D>;
  const int64_t blocks = (rows + C::kRows - 1) / C::kRows;
  if (blocks > 0x7fffffffLL) return cudaErrorInvalidValue;
  // programmatic launch: starts while the check kernel before it finishes
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const auto fn = wide ? rope_int4_append_kernel<D, true> : rope_int4_append_kernel<D, false>;
  const int quarters = append_prefetch_quarters();
  if (quarters > 0) {
    int64_t resident = 0;
    const cudaError_t e = resident_ctas(reinterpret_cast<const void*>(fn), C::kThreads, 0, &resident);
    if (e != cudaSuccess) return e;
    q.prefetch_rows = quarters * resident / 4 * C::kRows;
  }
  cfg.gridDim = dim3(static_cast<unsigned>(blocks));
  cfg.blockDim = dim3(C::kThreads);
  cfg.dynamicSmemBytes = 0;
  return cudaLaunchKernelEx(&cfg, fn, q);
}

}  // namespace iris

using namespace iris;

static bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

extern "C" size_t iris_b200_append_check_workspace_bytes(int64_t num_pages, int32_t page_size) {
  if (num_pages < 0 || page_size <= 0) return 0;
  const int64_t slots = num_pages * page_size;
  return static_cast<size_t>(((slots + 31) / 32) * 4);
}

extern "C" int iris_b200_append_check(const int32_t* positions, const int32_t* slot_mapping, int64_t num_tokens,
                                      int64_t max_position, int64_t num_pages, int32_t page_size, void* workspace,
                                      size_t workspace_bytes, int32_t* error_word, void* stream) {
  if (num_tokens < 0 || num_pages < 0 || page_size <= 0 || error_word == nullptr) return IRIS_EINVAL;
  if (num_tokens == 0) return IRIS_OK;
  if (positions == nullptr || slot_mapping == nullptr) return IRIS_EINVAL;
  const size_t need = iris_b200_append_check_workspace_bytes(num_pages, page_size);
  if (workspace_bytes < need || (need > 0 && workspace == nullptr)) return IRIS_EWORKSPACE;
  if (!aligned(workspace, 4)) return IRIS_EALIGN;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  clear_stale_cuda_error();
  if (need > 0) {
    const cudaError_t e = cudaMemsetAsync(workspace, 0, need, s);
    if (e != cudaSuccess) {
      record_cuda_error(e, "cudaMemsetAsync(slot bitmap)");
      return IRIS_ECUDA;
    }
  }
  const int threads = 256;
  const int64_t blocks = (num_tokens + threads - 1) / threads;
  append_check_kernel<<<static_cast<unsigned>(blocks), threads, 0, s>>>(
      positions, slot_mapping, num_tokens, max_position, num_pages * page_size, static_cast<uint32_t*>(workspace),
      error_word);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    record_cuda_error(e, "append_check_kernel launch");
    return IRIS_ECUDA;
  }
  return IRIS_OK;
}

extern "C" int iris_b200_rope_int4_paged_append(const void* key, const void* value, const int32_t* positions,
                                                const int32_t* slot_mapping, const void* cos_cache,
                                                const void* sin_cache, void* k_data, void* v_data, void* k_scale,
                                                void* v_scale, int64_t num_tokens, int32_t num_kv_heads,
                                                int32_t head_dim, int64_t max_position, int64_t num_pages,
                                                int32_t page_size, int32_t* error_word, void* stream) {
  if (num_tokens < 0 || num_kv_heads <= 0 || page_size <= 0 || num_pages < 0 || max_position < 0)
    return IRIS_EINVAL;
  if (head_dim <= 0 || head_dim % 64 != 0 || head_dim > 512) return IRIS_EUNSUPPORTED;
  if (num_tokens == 0) return IRIS_OK;
  if (num_tokens * num_kv_heads >= (1ll << 31) || num_pages * page_size >= (1ll << 31)) return IRIS_EUNSUPPORTED;
  const void* ptrs[] = {key, value, positions, slot_mapping, cos_cache, sin_cache, k_data, v_data, k_scale, v_scale};
  for (const void* q : ptrs)
    if (q == nullptr) return IRIS_EINVAL;
  if (!aligned(key, 16) || !aligned(value, 16) || !aligned(cos_cache, 16) || !aligned(sin_cache, 16) ||
      !aligned(k_data, 16) || !aligned(v_data, 16) || !aligned(k_scale, 2) || !aligned(v_scale, 2))
    return IRIS_EALIGN;
  AppendParams p = {};
  p.key = static_cast<const __half*>(key);
  p.value = static_cast<const __half*>(value);
  p.positions = positions;
  p.slots = slot_mapping;
  p.cos_cache = static_cast<const __half*>(cos_cache);
  p.sin_cache = static_cast<const __half*>(sin_cache);
  p.k_data = static_cast<uint8_t*>(k_data);
  p.v_data = static_cast<uint8_t*>(v_data);
  p.k_scale = static_cast<__half*>(k_scale);
  p.v_scale = static_cast<__half*>(v_scale);
  p.num_tokens = num_tokens;
  p.max_position = max_position;
  p.num_slots = num_pages * page_size;
  p.num_heads = num_kv_heads;
  p.page_size = page_size;
  p.heads_div = FastDiv::make(static_cast<uint32_t>(num_kv_heads));
  p.page_div = FastDiv::make(static_cast<uint32_t>(page_size));
  p.err = error_word;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  clear_stale_cuda_error();
  cudaError_t e;
  switch (head_dim) {
    case 64: e = launch_append<64>(p, s); break;
    case 128: e = launch_append<128>(p, s); break;
    case 192: e = launch_append<192>(p, s); break;
    case 256: e = launch_append<256>(p, s); break;
    case 320: e = launch_append<320>(p, s); break;
    case 384: e = launch_append<384>(p, s); break;
    case 448: e = launch_append<448>(p, s); break;
    default: e = launch_append<512>(p, s); break;
  }
  if (e != cudaSuccess) {
    record_cuda_error(e, "rope_int4_append_kernel launch");
    return IRIS_ECUDA;
  }
  return IRIS_OK;
}

extern "C" int iris_b200_int4_quantize_pack(const void* x, void* packed, void* scales, int64_t rows, int32_t head_dim,
                                            void* stream) {
  if (rows < 0 || head_dim <= 0 || head_dim % 32 != 0) return IRIS_EINVAL;
  if (rows == 0) return IRIS_OK;
  if (x == nullptr || packed == nullptr || scales == nullptr) return IRIS_EINVAL;
  if (!aligned(x, 16) || !aligned(packed, 16) || !aligned(scales, 2)) return IRIS_EALIGN;
  const int64_t groups = rows * (head_dim / 32);
  const int threads = 256;
  const int64_t blocks = (groups + threads - 1) / threads;
  if (blocks > 0x7fffffffLL) return IRIS_EUNSUPPORTED;
  clear_stale_cuda_error();
  quantize_pack_kernel<<<static_cast<unsigned>(blocks), threads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __half*>(x), static_cast<uint8_t*>(packed), static_cast<__half*>(scales), groups);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    record_cuda_error(e, "quantize_pack_kernel launch");
    return IRIS_ECUDA;
  }
  return IRIS_OK;
}

extern "C" int iris_b200_rope_fp16_paged_append(const void* key, const void* value, const int32_t* positions,
                                                const int32_t* slot_mapping, const void* cos_cache,
                                                const void* sin_cache, void* k_cache, void* v_cache,
                                                int64_t num_tokens, int32_t num_kv_heads, int32_t head_dim,
                                                int32_t rotary_dim, int64_t max_position, int64_t num_pages,
                                                int32_t page_size, int32_t* error_word, void* stream) {
  if (num_tokens < 0 || num_kv_heads <= 0 || head_dim <= 0 || page_size <= 0 || num_pages < 0) return IRIS_EINVAL;
  if (rotary_dim < 0 || rotary_dim > head_dim || rotary_dim % 2 != 0) return IRIS_EINVAL;
  if (num_tokens == 0) return IRIS_OK;
  const void* ptrs[] = {key, value, positions, slot_mapping, k_cache, v_cache};
  for (const void* q : ptrs)
    if (q == nullptr) return IRIS_EINVAL;
  if (rotary_dim > 0 && (cos_cache == nullptr || sin_cache == nullptr)) return IRIS_EINVAL;
  Fp16AppendParams p;
  p.key = static_cast<const __half*>(key);
  p.value = static_cast<const __half*>(value);
  p.positions = positions;
  p.slots = slot_mapping;
  p.cos_cache = static_cast<const __half*>(cos_cache);
  p.sin_cache = static_cast<const __half*>(sin_cache);
  p.k_cache = static_cast<__half*>(k_cache);
  p.v_cache = static_cast<__half*>(v_cache);
  p.num_tokens = num_tokens;
  p.max_position = max_position;
  p.num_slots = num_pages * page_size;
  p.num_heads = num_kv_heads;
  p.head_dim = head_dim;
  p.rotary_dim = rotary_dim;
  p.err = error_word;
  const bool vec = head_dim % 8 == 0 && rotary_dim % 16 == 0 && aligned(key, 16) && aligned(value, 16) &&
                   aligned(k_cache, 16) && aligned(v_cache, 16) && (rotary_dim == 0 || (aligned(cos_cache, 16) &&
                                                                                        aligned(sin_cache, 16)));
  // 32-byte loads when every row, partner and cos / sin chunk of 16 dims is 32-byte aligned
  const bool wide = vec && head_dim % 16 == 0 && rotary_dim % 32 == 0 && aligned(key, 32) && aligned(value, 32) &&
                    aligned(k_cache, 32) && aligned(v_cache, 32) &&
                    (rotary_dim == 0 || (aligned(cos_cache, 32) && aligned(sin_cache, 32))) && append_wide_enabled();
  const int width = wide ? 16 : vec ? 8 : 1;
  const int64_t threads_total = num_tokens * num_kv_heads * (head_dim / width);
  const int threads = 256;
  const int64_t blocks = (threads_total + threads - 1) / threads;
  if (blocks > 0x7fffffffLL) return IRIS_EUNSUPPORTED;
  const bool k32 = blocks * threads < (1LL << 31);
  p.row_div = FastDiv::make(static_cast<uint32_t>(head_dim / width));
  p.head_div = FastDiv::make(static_cast<uint32_t>(num_kv_heads));
  clear_stale_cuda_error();
  // programmatic launch: starts while the check kernel before it finishes
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(blocks));
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  const bool small = num_tokens <= kInlineCheckTokens;  // validated inside the kernel, ordinary launch
  cfg.numAttrs = small ? 0 : 1;
  const cudaError_t e = width == 16 ? launch_fp16_append<16>(cfg, p, small, k32)
                        : width == 8   ? launch_fp16_append<8>(cfg, p, small, k32)
                                       : launch_fp16_append<1>(cfg, p, small, k32);
  if (e != cudaSuccess) {
    record_cuda_error(e, "rope_fp16_append_kernel launch");
    return IRIS_ECUDA;
  }
  return IRIS_OK;
}

namespace {

// Exhaustive check of the division-free quantiser (group_scale +
// quant_pack_vec, the finite-scale path of every INT4 append) against the
// reference's arithmetic written with IEEE operations: scale =
// fp16(max(amax / 7, 2^-14)) with __fdiv_rn, q = clamp(rint(x / scale), -7, 7)
// with __fdiv_rn and __float2int_rn.  blockIdx.y selects the group absmax
// (non-negative finite fp16 bit pattern amax_lo + blockIdx.y); each thread
// takes 8 consecutive magnitudes x <= amax (both signs: every fp16 x with
// |x| <= amax is reachable in a group with that absmax) and compares the two
// packed words.  Magnitudes above amax are replaced by 0 (the same q = 0 on
// both paths).  counts[0] += mismatching words, counts[1] += amax values
// whose scale differs, counts[2] += words compared.
__global__ void __launch_bounds__(256) quantizer_sweep_kernel(uint32_t amax_lo, unsigned long long* counts) {
  const uint32_t amax_bits = amax_lo + blockIdx.y;
  const uint32_t m0 = 8u * (blockIdx.x * blockDim.x + threadIdx.x);
  const __half amax = __ushort_as_half(static_cast<unsigned short>(amax_bits));
  const __half s16 = iris::group_scale(amax);
  if (m0 == 0) {
    const float a = __half2float(amax);
    float s = __fdiv_rn(a, 7.0f);
    s = s < 6.103515625e-05f ? 6.103515625e-05f : s;
    if (__half_as_ushort(__float2half_rn(s)) != __half_as_ushort(s16)) atomicAdd(counts + 1, 1ull);
  }
  if (m0 > amax_bits) return;
  const float sc = __half2float(s16);
  const float r = iris::rcp_approx(sc);
  unsigned long long bad = 0;
#pragma unroll
  for (int sign = 0; sign < 2; ++sign) {
    uint4 raw;
    uint32_t* w = reinterpret_cast<uint32_t*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint32_t lo = m0 + 2 * i, hi = m0 + 2 * i + 1;
      lo = lo <= amax_bits ? lo | (sign << 15) : 0u;
      hi = hi <= amax_bits ? hi | (sign << 15) : 0u;
      w[i] = lo | (hi << 16);
    }
    const __half2* v = reinterpret_cast<const __half2*>(&raw);
    const __half2 vv[4] = {v[0], v[1], v[2], v[3]};
    bad += iris::quant_pack_vec(raw, sc, r) != iris::quant_pack8_ieee(vv, sc) ? 1ull : 0ull;
  }
  if (bad) atomicAdd(counts, bad);
  const unsigned active = __activemask();
  if ((threadIdx.x & 31) == __ffs(active) - 1) atomicAdd(counts + 2, 2ull * __popc(active));
}

}  // namespace

extern "C" int iris_b200_selftest_quantizer_sweep(int32_t amax_lo, int32_t amax_hi, unsigned long long* counts,
                                                  void* stream) {
  if (counts == nullptr || amax_lo < 0 || amax_hi > 0x7C00 || amax_lo >= amax_hi) return IRIS_EINVAL;
  clear_stale_cuda_error();
  const uint32_t n = static_cast<uint32_t>(amax_hi - amax_lo);
  // magnitudes 0 .. amax_hi - 1, 8 per thread
  const uint32_t threads = 256, per_block = 8 * threads;
  const dim3 grid((static_cast<uint32_t>(amax_hi) + per_block - 1) / per_block, n);
  quantizer_sweep_kernel<<<grid, threads, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<uint32_t>(amax_lo),
                                                                                 counts);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    record_cuda_error(e, "quantizer_sweep_kernel launch");
    return IRIS_ECUDA;
  }
  return IRIS_OK;
}
