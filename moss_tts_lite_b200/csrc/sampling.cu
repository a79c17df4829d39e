// Fused per-row token sampling for sm_100a: sample_token of the reference
// (moss_tts_lite/sampling.py:70-98) for one decode step of generate_fast
// (moss_tts_lite/fast.py:491-545), one CTA per logits row:
//
//   1. temperature:  x = bf16(x * (1/T))  (PyTorch on CUDA divides by a Python
//      scalar as a multiply by its float reciprocal), excluded ids -> -inf;
//   2. repetition penalty (sampling.py:36-67) on the ids of a device bitmap:
//      x > 0 ? bf16(x * (1/p)) : bf16(x * p);
//   3. top-k (sampling.py:9-17): the k largest by a two-pass radix select on
//      order-preserving bf16 keys; ties at the threshold keep the lowest ids;
//   4. top-p (sampling.py:101-113): bf16 softmax of the candidates, sorted
//      descending (ties by id), cumulative sum with every partial sum rounded
//      to bf16 and grouped as PyTorch's CUDA cumsum groups it for the shape
//      the reference scanned (scan_device_wide / scan_rows_sklansky below),
//      removal where cumsum > bf16(top_p) shifted by one (the top candidate
//      always stays);
//   5. multinomial (sampling.py:96-97): bf16 softmax of the survivors and one
//      categorical draw in id order from a Philox4x32-10 uniform (Salmon et
//      al., SC'11) keyed by (seed, offset, row).
//
// Rows of at least kSliceMinCols columns with a top-k (the text head's
// 151,936 logits) take two launches: sample_slices_kernel splits the row
// into slices of equal length (each at least top_k long), one CTA per slice,
// and writes each slice's top-k (value after steps 1-2, id) in id order;
// sample_rows_kernel<true> then runs steps 3-5 on the concatenated slice
// candidates.  The row's top-k is a subset of the union of the slices'
// top-k, and both selections keep the lowest ids among ties at the
// threshold, so the candidate set is the same as one pass over the row.
//
// The candidate set and its probabilities follow the reference's arithmetic;
// the random stream is this library's own (torch.multinomial's stream cannot
// be reproduced), so sampled tokens agree with the reference in
// distribution, and bit-exactly with oracle/sampling.py's restatement.
#include <algorithm>

#include "common.cuh"

namespace mtl {

constexpr int kSampleThreads = 512;
constexpr int kSampleMaxCand = 2048;
constexpr int kSampleMaxRows = 40;
constexpr int kSampleMaxExcl = 8;
constexpr int kSliceThreads = 256;
constexpr int kSliceMinCols = 16384;
constexpr int kSliceMaxLen = 8192;  // values of one slice in shared memory (32 KB)

struct SampleArgs {
  const uint16_t* logits;  // bf16, row r at logits + row_index[r] * ld
  int ld, cols, n_rows;
  int row_index[kSampleMaxRows];
  int seen_set[kSampleMaxRows];  // -1: no penalty for this row
  const uint32_t* seen_bits;     // [sets][words_per_set] (nullable)
  int words_per_set;
  float inv_temp, penalty, inv_penalty;
  int top_k;       // <= 0: no top-k
  float top_p_bf;  // top_p rounded to bf16; >= 1: no top-p
  int n_excl;
  int excl[kSampleMaxExcl];
  // grouping of the top-p cumsum per row: 0 = the reference scanned a one-row
  // tensor (device-wide scan), else log2 of the threads per row of the
  // shared-memory scan of a multi-row tensor
  int scan_lognx[kSampleMaxRows];
  uint32_t seed_lo, seed_hi, off_lo, off_hi;
  int64_t* out;
  int64_t out_add;  // added to the sampled column index
  // sliced path (slices > 0): row r's slice s writes top_k candidates at
  // cand_val/cand_id + (r * slices + s) * top_k
  int slices, slice_len;
  float* cand_val;
  int32_t* cand_id;
};

// Slices for a row of `cols` values and a top-k of `top_k`: every slice at
// least top_k long (the last one included) and at most kSliceMaxLen; 0 when
// the row is short, has no top-k, or cannot be cut that way.
inline int sample_slice_count(int cols, int top_k, int* slice_len) {
  if (cols < kSliceMinCols || top_k <= 0 || top_k >= cols) return 0;
  for (int ns = std::min(148, cols / std::max(top_k, 1024)); ns >= 2; --ns) {
    const int sl = (cols + ns - 1) / ns;
    if (sl > kSliceMaxLen) return 0;  // fewer slices only make them longer
    if (cols - (ns - 1) * sl >= top_k) {
      *slice_len = sl;
      return ns;
    }
  }
  return 0;
}

// Philox4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel random numbers: as
// easy as 1, 2, 3", SC 2011): 10 rounds of the 4x32 bijection with the
// published multipliers and Weyl key increments.
__device__ __forceinline__ void philox4x32_10(uint32_t c[4], uint32_t k0, uint32_t k1) {
  const uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u, W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t hi0 = __umulhi(M0, c[0]), lo0 = M0 * c[0];
    const uint32_t hi1 = __umulhi(M1, c[2]), lo1 = M1 * c[2];
    const uint32_t n0 = hi1 ^ c[1] ^ k0, n1 = lo1, n2 = hi0 ^ c[3] ^ k1, n3 = lo0;
    c[0] = n0;
    c[1] = n1;
    c[2] = n2;
    c[3] = n3;
    k0 += W0;
    k1 += W1;
  }
}

// Order-preserving 16-bit key of a bf16 value (larger value -> larger key).
__device__ __forceinline__ uint32_t bf16_key(uint16_t b) { return (b & 0x8000u) ? (uint32_t)(~b & 0xFFFFu) : (uint32_t)(b | 0x8000u); }

__device__ __forceinline__ float row_value(const SampleArgs& a, const uint16_t* row, int c, int set) {
  for (int e = 0; e < a.n_excl; ++e)
    if (a.excl[e] == c) return -INFINITY;
  float v = bf16_bits_to_f32(row[c]);
  if (a.inv_temp != 1.0f) v = round_bf16(v * a.inv_temp);
  if (set >= 0 && a.seen_bits && ((a.seen_bits[(size_t)set * a.words_per_set + (c >> 5)] >> (c & 31)) & 1u))
    v = (v > 0.f) ? round_bf16(v * a.inv_penalty) : round_bf16(v * a.penalty);
  return v;
}

// torch.cumsum of a one-row bf16 tensor on CUDA is CUB's device-wide
// inclusive scan with std::plus<c10::BFloat16> (fp32 add, round to bf16):
// thread t of a tile owns kCubItems consecutive items and reduces them left
// to right, warps scan the thread totals Kogge-Stone style, warps chain left
// to right within a tile of kCubTileThreads threads, tiles chain left to
// right, and each thread adds its items one by one onto its exclusive
// prefix.  Thread t here plays that scan's thread t (so warps coincide).
// cs[0, nc) holds the sorted probabilities on entry, the scan on exit;
// cs[nc, kSampleMaxCand) must be zero.
constexpr int kCubItems = 30;
constexpr int kCubTileThreads = 128;

__device__ void scan_device_wide(float* cs, int nc, float* wagg) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nthr = (nc + kCubItems - 1) / kCubItems;  // <= 69 for 2048 items
  const int nwarps = (nthr + 31) / 32;
  float agg = 0.f;
  if (tid < nthr) {
    const float* it = cs + tid * kCubItems;
    agg = it[0];
    for (int i = 1; i < kCubItems; ++i)
      if (tid * kCubItems + i < kSampleMaxCand) agg = round_bf16(agg + it[i]);
  }
  float inc = agg;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const float up = __shfl_up_sync(0xFFFFFFFFu, inc, off);
    if (lane >= off) inc = round_bf16(up + inc);
  }
  float exc = __shfl_up_sync(0xFFFFFFFFu, inc, 1);
  if (lane == 0) exc = 0.f;  // exactly "no prefix": bf16(0 + x) == x
  if (lane == 31 && warp < nwarps) wagg[warp] = inc;
  __syncthreads();
  if (tid < nthr) {
    // warp prefix inside the tile, tile prefix from the chain of tile totals
    const int wpt = kCubTileThreads / 32, t0 = (warp / wpt) * wpt;
    float tile_prefix = 0.f;
    for (int tw = 0; tw < t0; tw += wpt) {
      float ba = wagg[tw];
      for (int w = tw + 1; w < tw + wpt && w < nwarps; ++w) ba = round_bf16(ba + wagg[w]);
      tile_prefix = tw == 0 ? ba : round_bf16(tile_prefix + ba);
    }
    if (warp > t0) {
      float wp = wagg[t0];
      for (int w = t0 + 1; w < warp; ++w) wp = round_bf16(wp + wagg[w]);
      exc = lane == 0 ? wp : round_bf16(wp + exc);
    }
    if (t0 > 0) exc = round_bf16(tile_prefix + exc);
    float run = exc;
    float* it = cs + tid * kCubItems;
    for (int i = 0; i < kCubItems && tid * kCubItems + i < kSampleMaxCand; ++i) {
      run = round_bf16(run + it[i]);
      it[i] = run;
    }
  }
  __syncthreads();
}

// torch.cumsum of each row of a multi-row bf16 tensor on CUDA
// (tensor_kernel_scan_innermost_dim): chunks of 2 * 2^lognx items, the total
// of the earlier chunks added onto the chunk's first item, then lognx + 1
// Sklansky rounds; round m adds item a - 1 onto items a + j (j < 2^m) with
// a = (x >> m << (m + 1)) | 2^m for x < 2^lognx.  In place on cs[0, nc);
// cs[nc, kSampleMaxCand) must be zero (2 * 2^lognx divides kSampleMaxCand).
__device__ void scan_rows_sklansky(float* cs, int nc, int lognx) {
  const int tid = threadIdx.x, nx = 1 << lognx;
  float carry = 0.f;
  for (int base = 0; base < nc; base += 2 * nx) {
    if (tid == 0) cs[base] = round_bf16(cs[base] + carry);
    __syncthreads();
    for (int m = 0; m <= lognx; ++m) {
      for (int x = tid; x < nx; x += kSampleThreads) {
        const int sz = 1 << m;
        const int a = ((x >> m) << (m + 1)) | sz;
        const int ti = a + (x & (sz - 1)), si = a - 1;
        cs[base + ti] = round_bf16(cs[base + ti] + cs[base + si]);
      }
      __syncthreads();
    }
    carry = cs[base + 2 * nx - 1];
    __syncthreads();
  }
}

// Radix-select step over a 256-bin histogram: the largest b in [1, 255] with
// S(b) = sum_{b' >= b} hist[b'] >= need (0 if there is none), and how many
// are still needed from bin b: out[0] = b, out[1] = need - S(b + 1).  The bin
// totals are suffix-scanned by the first 256 threads; every thread of the
// block calls this (blockDim.x a multiple of 32 and >= 256).
__device__ void select_bin(const unsigned* hist, int need, int* out, int* wsum) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int b = 255 - tid;
  const int v = tid < 256 ? (int)hist[b] : 0;
  int inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int u = __shfl_up_sync(0xFFFFFFFFu, inc, o);
    if (lane >= o) inc += u;
  }
  __syncthreads();  // wsum may still be read by an earlier call
  if (tid < 256 && lane == 31) wsum[warp] = inc;
  __syncthreads();
  if (tid < 256) {
    int pre = 0;
    for (int w = 0; w < warp; ++w) pre += wsum[w];
    const int S = pre + inc, Snext = S - v;
    if (b >= 1 && S >= need && Snext < need) {
      out[0] = b;
      out[1] = need - Snext;
    }
    if (b == 1 && S < need) {
      out[0] = 0;
      out[1] = need - S;
    }
  }
  __syncthreads();
}

// Exclusive block-wide prefix sum of x; *total = the sum over the block.
__device__ int block_excl_scan(int x, int* wsum, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  int inc = x;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int u = __shfl_up_sync(0xFFFFFFFFu, inc, o);
    if (lane >= o) inc += u;
  }
  __syncthreads();
  if (lane == 31) wsum[warp] = inc;
  __syncthreads();
  int pre = 0, tot = 0;
  for (int w = 0; w < nw; ++w) {
    const int t = wsum[w];
    if (w < warp) pre += t;
    tot += t;
  }
  *total = tot;
  return pre + inc - x;
}

// One CTA per (slice, row): the slice's top_k largest values after
// temperature, exclusions and penalty (ties at the threshold: lowest ids),
// written in id order.
__global__ void __launch_bounds__(kSliceThreads) sample_slices_kernel(const SampleArgs a) {
  extern __shared__ float sv[];  // the slice's values
  __shared__ unsigned hist[kSliceThreads / 32][256];
  __shared__ int wsum[kSliceThreads / 32];
  __shared__ int sel[2];
  pdl_launch_dependents();
  pdl_wait();
  const int sl = blockIdx.x, r = blockIdx.y, tid = threadIdx.x, warp = tid >> 5;
  const uint16_t* row = a.logits + (size_t)a.row_index[r] * a.ld;
  const int set = a.seen_set[r];
  const int lo = sl * a.slice_len, len = min(a.cols, lo + a.slice_len) - lo;
  const int k = a.top_k;  // 0 < k <= len (host)
  for (int i = tid; i < len; i += kSliceThreads) sv[i] = row_value(a, row, lo + i, set);
  uint32_t prefix = 0;
  int need = k;
  for (int pass = 0; pass < 2; ++pass) {
    const int shift = pass == 0 ? 8 : 0;
    for (int i = tid; i < (kSliceThreads / 32) * 256; i += kSliceThreads) (&hist[0][0])[i] = 0;
    __syncthreads();
    for (int i = tid; i < len; i += kSliceThreads) {
      const uint32_t key = bf16_key(f32_to_bf16_bits(sv[i]));
      if (pass == 0 || (key >> 8) == (prefix >> 8)) atomicAdd(&hist[warp][(key >> shift) & 0xFFu], 1u);
    }
    __syncthreads();
    for (int b = tid; b < 256; b += kSliceThreads) {
      unsigned t = 0;
      for (int w = 0; w < kSliceThreads / 32; ++w) t += hist[w][b];
      hist[0][b] = t;
    }
    __syncthreads();
    select_bin(&hist[0][0], need, sel, wsum);
    prefix |= (uint32_t)sel[0] << shift;
    need = sel[1];
  }
  const uint32_t thr = prefix;
  const int take_eq = need;
  const int per = (len + kSliceThreads - 1) / kSliceThreads;
  const int i0 = min(len, tid * per), i1 = min(len, i0 + per);
  int my_gt = 0, my_eq = 0;
  for (int i = i0; i < i1; ++i) {
    const uint32_t key = bf16_key(f32_to_bf16_bits(sv[i]));
    if (key > thr) ++my_gt;
    else if (key == thr) ++my_eq;
  }
  int tot;
  const int eq_before = block_excl_scan(my_eq, wsum, &tot);
  int eq_left = max(0, min(my_eq, take_eq - eq_before));
  int w = block_excl_scan(my_gt + eq_left, wsum, &tot);
  float* ov = a.cand_val + ((size_t)r * a.slices + sl) * k;
  int32_t* oi = a.cand_id + ((size_t)r * a.slices + sl) * k;
  for (int i = i0; i < i1 && w < k; ++i) {
    const uint32_t key = bf16_key(f32_to_bf16_bits(sv[i]));
    bool keep = key > thr;
    if (!keep && key == thr && eq_left > 0) {
      keep = true;
      --eq_left;
    }
    if (keep) {
      ov[w] = sv[i];
      oi[w] = lo + i;
      ++w;
    }
  }
}

// CAND: read the row as the slices' candidates (values final, ids listed).
template <bool CAND>
__global__ void __launch_bounds__(kSampleThreads) sample_rows_kernel(const SampleArgs a) {
  __shared__ float cv[kSampleMaxCand];    // candidate values (in id order)
  __shared__ int ci[kSampleMaxCand];      // candidate ids
  __shared__ float cp[kSampleMaxCand];    // probabilities
  __shared__ int order[kSampleMaxCand];   // candidate slots sorted by probability
  __shared__ float cs[kSampleMaxCand];    // cumulative sum over the sorted order
  __shared__ unsigned hist[256];
  __shared__ int scan[kSampleThreads];
  __shared__ float fred[kSampleThreads / 32];
  __shared__ int sh_int[4];
  __shared__ int wsum[kSampleThreads / 32];
  pdl_launch_dependents();
  pdl_wait();
  const int r = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint16_t* row = a.logits + (size_t)a.row_index[r] * a.ld;
  const int set = a.seen_set[r];
  const int n = CAND ? a.slices * a.top_k : a.cols;
  const float* cand_v = CAND ? a.cand_val + (size_t)r * n : nullptr;
  const int32_t* cand_i = CAND ? a.cand_id + (size_t)r * n : nullptr;
  auto value = [&](int c) { return CAND ? cand_v[c] : row_value(a, row, c, set); };
  // ---- threshold of the top-k (key of the k-th largest), radix select on 16 bits
  int k = (a.top_k > 0 && a.top_k < n) ? a.top_k : n;
  uint32_t thr = 0;  // candidates: key > thr, plus (k - count_gt) with key == thr in id order
  int take_eq = 0;
  if (k < n) {
    uint32_t prefix = 0;
    int need = k;  // how many of the remaining still have to be taken from the top
    for (int pass = 0; pass < 2; ++pass) {
      const int shift = pass == 0 ? 8 : 0;
      for (int i = tid; i < 256; i += kSampleThreads) hist[i] = 0;
      __syncthreads();
      for (int c = tid; c < n; c += kSampleThreads) {
        const uint32_t key = bf16_key(f32_to_bf16_bits(value(c)));
        if (pass == 0 || (key >> 8) == (prefix >> 8)) atomicAdd(&hist[(key >> shift) & 0xFFu], 1u);
      }
      __syncthreads();
      select_bin(hist, need, sh_int, wsum);  // sh_int[1]: still needed from bin sh_int[0]
      prefix |= (uint32_t)sh_int[0] << shift;
      need = sh_int[1];
    }
    thr = prefix;
    take_eq = need;  // elements with key == thr to take (lowest ids first)
  }
  // ---- collect candidates in id order: each thread owns a contiguous slice
  const int per = (n + kSampleThreads - 1) / kSampleThreads;
  const int c0 = min(n, tid * per), c1 = min(n, c0 + per);
  int my_gt = 0, my_eq = 0;
  for (int c = c0; c < c1; ++c) {
    const uint32_t key = bf16_key(f32_to_bf16_bits(value(c)));
    if (k == n || key > thr) ++my_gt;
    else if (key == thr) ++my_eq;
  }
  // exclusive scans of the "equal" counts (to take the lowest ids) and of the kept counts
  scan[tid] = my_eq;
  __syncthreads();
  for (int o = 1; o < kSampleThreads; o <<= 1) {
    const int v = tid >= o ? scan[tid - o] : 0;
    __syncthreads();
    scan[tid] += v;
    __syncthreads();
  }
  const int eq_before = scan[tid] - my_eq;
  const int my_eq_take = (k == n) ? 0 : max(0, min(my_eq, take_eq - eq_before));
  __syncthreads();
  const int my_keep = my_gt + my_eq_take;
  scan[tid] = my_keep;
  __syncthreads();
  for (int o = 1; o < kSampleThreads; o <<= 1) {
    const int v = tid >= o ? scan[tid - o] : 0;
    __syncthreads();
    scan[tid] += v;
    __syncthreads();
  }
  const int total = scan[kSampleThreads - 1];
  int w = scan[tid] - my_keep;
  int eq_left = my_eq_take;
  if (total <= kSampleMaxCand) {
    for (int c = c0; c < c1; ++c) {
      const float v = value(c);
      const uint32_t key = bf16_key(f32_to_bf16_bits(v));
      bool keep = (k == n) || key > thr;
      if (!keep && key == thr && eq_left > 0) {
        keep = true;
        --eq_left;
      }
      if (keep) {
        cv[w] = v;
        ci[w] = CAND ? cand_i[c] : c;
        ++w;
      }
    }
  }
  __syncthreads();
  if (total > kSampleMaxCand) {  // host validation prevents this; stay safe
    if (tid == 0) {
      flag_error(kDevBadIndex);
      a.out[r] = a.out_add;
    }
    return;
  }
  const int nc = total;
  // ---- softmax of the candidates (fp32 statistics, bf16 probabilities)
  auto softmax_bf16 = [&](void) {
    float mx = -INFINITY;
    for (int i = tid; i < nc; i += kSampleThreads) mx = fmaxf(mx, cv[i]);
    mx = warp_max(mx);
    if (lane == 0) fred[warp] = mx;
    __syncthreads();
    mx = fred[0];
    for (int i = 1; i < kSampleThreads / 32; ++i) mx = fmaxf(mx, fred[i]);
    __syncthreads();
    float s = 0.f;
    for (int i = tid; i < nc; i += kSampleThreads) s += (cv[i] == -INFINITY) ? 0.f : expf(cv[i] - mx);
    s = warp_sum(s);
    if (lane == 0) fred[warp] = s;
    __syncthreads();
    s = 0.f;
    for (int i = 0; i < kSampleThreads / 32; ++i) s += fred[i];
    for (int i = tid; i < nc; i += kSampleThreads) cp[i] = (cv[i] == -INFINITY) ? 0.f : round_bf16(expf(cv[i] - mx) / s);
    __syncthreads();
  };
  if (a.top_p_bf < 1.0f && nc > 1) {
    softmax_bf16();
    // sort slots by (probability desc, id asc): rank by counting (nc <= 2048)
    for (int i = tid; i < nc; i += kSampleThreads) {
      const float pi = cp[i];
      int rank = 0;
      for (int j = 0; j < nc; ++j) {
        const float pj = cp[j];
        rank += (pj > pi) || (pj == pi && j < i);
      }
      order[rank] = i;
    }
    __syncthreads();
    for (int s = tid; s < kSampleMaxCand; s += kSampleThreads) cs[s] = s < nc ? cp[order[s]] : 0.f;
    __syncthreads();
    if (a.scan_lognx[r] == 0)
      scan_device_wide(cs, nc, fred);
    else
      scan_rows_sklansky(cs, nc, a.scan_lognx[r]);
    // remove where cumsum > top_p, shifted by one so the first sorted
    // candidate stays
    for (int s = tid + 1; s < nc; s += kSampleThreads)
      if (cs[s - 1] > a.top_p_bf) cv[order[s]] = -INFINITY;
    __syncthreads();
  }
  softmax_bf16();
  // ---- one categorical draw in id order
  if (tid == 0) {
    uint32_t ctr[4] = {a.off_lo, a.off_hi, (uint32_t)r, 0u};
    philox4x32_10(ctr, a.seed_lo, a.seed_hi);
    const float u = (float)(ctr[0] >> 8) * (1.0f / 16777216.0f);
    float tot = 0.f;
    for (int i = 0; i < nc; ++i) tot += cp[i];
    int pick = -1;
    if (tot > 0.f) {
      const float target = u * tot;
      float run = 0.f;
      for (int i = 0; i < nc; ++i) {
        run += cp[i];
        if (cp[i] > 0.f && run > target) {
          pick = i;
          break;
        }
      }
      if (pick < 0)  // rounding at the very top: last candidate with mass
        for (int i = nc - 1; i >= 0; --i)
          if (cp[i] > 0.f) {
            pick = i;
            break;
          }
    }
    if (pick < 0) {  // no mass at all: first maximum
      float best = -INFINITY;
      for (int i = 0; i < nc; ++i)
        if (cv[i] > best) {
          best = cv[i];
          pick = i;
        }
      if (pick < 0) pick = 0;
    }
    a.out[r] = (nc > 0 ? (int64_t)ci[pick] : 0) + a.out_add;
  }
}

cudaError_t launch_sample_rows(const SampleArgs& a, cudaStream_t s) {
  if (a.slices > 0) {
    sample_slices_kernel<<<dim3(a.slices, a.n_rows), kSliceThreads, (size_t)a.slice_len * sizeof(float), s>>>(a);
    sample_rows_kernel<true><<<a.n_rows, kSampleThreads, 0, s>>>(a);
  } else {
    sample_rows_kernel<false><<<a.n_rows, kSampleThreads, 0, s>>>(a);
  }
  return cudaGetLastError();
}

}  // namespace mtl
