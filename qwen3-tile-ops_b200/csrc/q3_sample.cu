// Sampling after the lm_head on the device: tools/engine.py:118-149
// (Sampler.sample) for every row of a logits matrix, one CTA per row.
//
// The float64 steps are the reference's: x = logits / T (IEEE division), the
// repetition penalty on the row's generated ids, top-k as a threshold at the
// k-th largest value, top-p over the descending order, and the draw
// Generator.choice(V, p) = the first index whose cumulative probability
// exceeds the uniform u.  Order statistics are found without sorting:
//  * every float64 x maps to a 64-bit key with the same order (sign bit
//    flipped for x >= 0, all bits flipped for x < 0);
//  * top-k: radix select over the keys (8 levels of 256 buckets; each level
//    counts the elements under the current prefix and descends into the
//    bucket that holds the k-th largest);
//  * top-p: the same descent weighted by exp(x - max): buckets are taken from
//    the top while the running mass / total stays <= top_p, the descent ends at
//    the single key value where it crosses, and of the elements holding that
//    value the first r in index order are kept (r from the remaining mass);
//  * the draw: 16 warps own contiguous index segments; segment sums of the
//    kept masses, a scan over the segments, and the segment holding u * total
//    is scanned element by element.
// The row's x and exp(x - max) live in a float64 workspace (2 x vocab per row).
#include <math.h>
#include <stdint.h>

#include "q3_common.cuh"
#include "q3_rng.h"

namespace {

constexpr int kT = 512;           // threads per row
constexpr int kW = kT / 32;
constexpr int kB = 8;             // loads a thread issues before using them
constexpr int kCap = 4096;        // bucket size from which a descent continues in shared memory

__device__ __forceinline__ uint64_t okey(double x) {
  const uint64_t b = static_cast<uint64_t>(__double_as_longlong(x));
  return (b >> 63) ? ~b : (b | 0x8000000000000000ull);
}

struct Shared {
  uint32_t hc[256];
  double hm[256];
  double red_v[kW];
  int red_i[kW];
  double seg[kW];
  uint32_t tie_cnt[kW], tie_base[kW];
  uint64_t prefix, pmask;
  uint32_t need, ccount;
  int compact;
  double above;
  int digit, stop;
  double m;
  int amax;
  double total;
  uint64_t kkey, t_ge, t_tie;
  uint32_t r_ties;
  int pick_warp;
  double pick_base;
};

// first maximum (value, lowest index) over the block; every thread gets it
__device__ void block_argmax(double v, int i, Shared &sm, double &bv, int &bi) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const double ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, i, o);
    if (oi >= 0 && (i < 0 || ov > v || (ov == v && oi < i))) { v = ov; i = oi; }
  }
  if (lane == 0) { sm.red_v[w] = v; sm.red_i[w] = i; }
  __syncthreads();
  if (threadIdx.x == 0) {
    double b = sm.red_v[0];
    int bix = sm.red_i[0];
    for (int k = 1; k < kW; ++k) {
      const double ov = sm.red_v[k];
      const int oi = sm.red_i[k];
      if (oi >= 0 && (bix < 0 || ov > b || (ov == b && oi < bix))) { b = ov; bix = oi; }
    }
    sm.m = b;
    sm.amax = bix;
  }
  __syncthreads();
  bv = sm.m;
  bi = sm.amax;
}

__device__ double block_sum(double v, Shared &sm) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if (lane == 0) sm.red_v[w] = v;
  __syncthreads();
  if (threadIdx.x == 0) {
    double s = 0.0;
    for (int k = 0; k < kW; ++k) s += sm.red_v[k];
    sm.total = s;
  }
  __syncthreads();
  return sm.total;
}

// the candidates of a descent once they fit in shared memory
struct Cand {
  uint64_t *key;
  double *e;
};

// one level of the descent: counts (and masses) of the elements under
// (prefix, pmask) per 8-bit digit at `shift`, over the row or, once
// compacted, over the shared candidates; runs of equal digits in a thread's
// elements are added to the shared histogram once
__device__ void histogram(const double *X, const double *E, int V, int shift, Shared &sm,
                          Cand c) {
  for (int d = threadIdx.x; d < 256; d += kT) { sm.hc[d] = 0; sm.hm[d] = 0.0; }
  __syncthreads();
  const uint64_t prefix = sm.prefix, pmask = sm.pmask;
  int cur = -1;
  uint32_t cnt = 0;
  double mass = 0.0;
  if (sm.compact) {
    for (uint32_t j = threadIdx.x; j < sm.ccount; j += kT) {
      const uint64_t key = c.key[j];
      if ((key & pmask) != prefix) continue;
      const int d = static_cast<int>((key >> shift) & 255u);
      atomicAdd(&sm.hc[d], 1u);
      if (E) atomicAdd(&sm.hm[d], c.e[j]);
    }
    __syncthreads();
    return;
  }
  for (int base = threadIdx.x; base < V; base += kB * kT) {
    double xv[kB], ev[kB];
#pragma unroll
    for (int j = 0; j < kB; ++j) {
      const int i = base + j * kT;
      xv[j] = i < V ? X[i] : 0.0;
      ev[j] = (E && i < V) ? E[i] : 0.0;
    }
#pragma unroll
    for (int j = 0; j < kB; ++j) {
      if (base + j * kT >= V) break;
      const uint64_t key = okey(xv[j]);
      if ((key & pmask) != prefix) continue;
      const int d = static_cast<int>((key >> shift) & 255u);
      if (d != cur) {
        if (cnt) {
          atomicAdd(&sm.hc[cur], cnt);
          if (E) atomicAdd(&sm.hm[cur], mass);
        }
        cur = d;
        cnt = 0;
        mass = 0.0;
      }
      ++cnt;
      mass += ev[j];
    }
  }
  if (cnt) {
    atomicAdd(&sm.hc[cur], cnt);
    if (E) atomicAdd(&sm.hm[cur], mass);
  }
  __syncthreads();
}

// after a level: when the chosen bucket fits, copy its elements (key, mass)
// into shared memory; later levels read them there
__device__ void maybe_compact(const double *X, const double *E, int V, uint32_t count, Shared &sm,
                              Cand c) {
  if (sm.compact || count > static_cast<uint32_t>(kCap)) return;
  const uint64_t prefix = sm.prefix, pmask = sm.pmask;
  for (int base = threadIdx.x; base < V; base += kB * kT) {
    double xv[kB];
#pragma unroll
    for (int j = 0; j < kB; ++j) xv[j] = base + j * kT < V ? X[base + j * kT] : 0.0;
#pragma unroll
    for (int j = 0; j < kB; ++j) {
      const int i = base + j * kT;
      if (i >= V) break;
      const uint64_t key = okey(xv[j]);
      if ((key & pmask) != prefix) continue;
      const uint32_t slot = atomicAdd(&sm.ccount, 1u);
      if (slot < static_cast<uint32_t>(kCap)) {
        c.key[slot] = key;
        c.e[slot] = E ? E[i] : 0.0;
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) sm.compact = 1;
  __syncthreads();
}

// key of the k-th largest x (np.partition(x, -k)[-k])
__device__ uint64_t kth_key(const double *X, int V, uint32_t k, Shared &sm, Cand c) {
  if (threadIdx.x == 0) { sm.prefix = 0; sm.pmask = 0; sm.need = k; sm.compact = 0; sm.ccount = 0; }
  __syncthreads();
  for (int shift = 56; shift >= 0; shift -= 8) {
    histogram(X, nullptr, V, shift, sm, c);
    if (threadIdx.x == 0) {
      uint32_t acc = 0;
      int d = 255;
      for (; d > 0; --d) {
        if (acc + sm.hc[d] >= sm.need) break;
        acc += sm.hc[d];
      }
      sm.need -= acc;
      sm.prefix |= static_cast<uint64_t>(d) << shift;
      sm.pmask |= 255ull << shift;
      sm.digit = d;
    }
    __syncthreads();
    if (shift) maybe_compact(X, nullptr, V, sm.hc[sm.digit], sm, c);
  }
  return sm.prefix;
}

// top-p boundary: keep key >= t_ge, plus the first r_ties (index order) of
// the elements whose key is t_tie
__device__ void top_p_bound(const double *X, const double *E, int V, double S, double top_p,
                            double m, Shared &sm, Cand c) {
  if (threadIdx.x == 0) {
    sm.prefix = 0;
    sm.pmask = 0;
    sm.above = 0.0;
    sm.stop = 0;
    sm.compact = 0;
    sm.ccount = 0;
  }
  __syncthreads();
  for (int shift = 56; shift >= 0; shift -= 8) {
    histogram(X, E, V, shift, sm, c);
    if (threadIdx.x == 0) {
      int d = 255, found = 0;
      double above = sm.above;
      for (; d >= 0; --d) {
        if (sm.hc[d] == 0) continue;
        if ((above + sm.hm[d]) / S <= top_p) { above += sm.hm[d]; continue; }
        found = 1;
        break;
      }
      if (!found) {
        // every element under the prefix stays (the crossing fell on the
        // prefix's last element by rounding): keep key >= prefix
        sm.t_ge = sm.prefix;
        sm.t_tie = 0;
        sm.r_ties = 0;
        sm.stop = 1;
      } else {
        sm.above = above;
        sm.prefix |= static_cast<uint64_t>(d) << shift;
        sm.pmask |= 255ull << shift;
        sm.digit = d;
      }
    }
    __syncthreads();
    if (sm.stop) return;
    if (shift) maybe_compact(X, E, V, sm.hc[sm.digit], sm, c);
  }
  if (threadIdx.x == 0) {
    // one key value: c equal elements of mass e_c; keep the first r
    const uint64_t kc = sm.prefix;
    const uint32_t c = sm.hc[sm.digit];
    const uint64_t b = (kc >> 63) ? (kc & 0x7FFFFFFFFFFFFFFFull) : ~kc;
    const double ec = exp(__longlong_as_double(static_cast<long long>(b)) - m);
    const double above = sm.above;
    double est = ec > 0.0 ? floor((top_p * S - above) / ec) : 0.0;
    uint32_t r = est <= 0.0 ? 0u : (est >= static_cast<double>(c) ? c : static_cast<uint32_t>(est));
    while (r < c && (above + static_cast<double>(r + 1) * ec) / S <= top_p) ++r;
    while (r > 0 && (above + static_cast<double>(r) * ec) / S > top_p) --r;
    sm.t_ge = kc + 1;
    sm.t_tie = kc;
    sm.r_ties = r;
  }
  __syncthreads();
}

__global__ void __launch_bounds__(kT, 1)
    k_sample_rows(const float *logits, long long stride, int V, const q3_sample_row *params,
                  const int32_t *generated, int32_t *out, double *ws) {
  extern __shared__ uint32_t bitmap[];
  __shared__ Shared sm;
  const int r = blockIdx.x, tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const q3_sample_row p = params[r];
  const float *lg = logits + static_cast<long long>(r) * stride;

  if (!(p.temperature > 0.0)) {   // np.argmax: the first maximum
    double bv = -INFINITY;
    int bi = -1;
    for (int base = tid; base < V; base += kB * kT) {
      float lv[kB];
#pragma unroll
      for (int j = 0; j < kB; ++j) lv[j] = base + j * kT < V ? lg[base + j * kT] : 0.0f;
#pragma unroll
      for (int j = 0; j < kB; ++j) {
        const int i = base + j * kT;
        const double v = static_cast<double>(lv[j]);
        if (i < V && (bi < 0 || v > bv)) { bv = v; bi = i; }
      }
    }
    double m;
    int a;
    block_argmax(bv, bi, sm, m, a);
    if (tid == 0) out[r] = a;
    return;
  }

  double *X = ws + static_cast<size_t>(r) * 2 * V;
  double *E = X + V;
  const int nb = (V + 31) >> 5;
  Cand cand;
  cand.key = reinterpret_cast<uint64_t *>(bitmap + ((nb + 1) & ~1));
  cand.e = reinterpret_cast<double *>(cand.key + kCap);
  const bool pen = p.repetition_penalty != 1.0;
  if (pen) {
    for (int j = tid; j < nb; j += kT) bitmap[j] = 0;
    __syncthreads();
    for (uint32_t j = tid; j < p.gen_count; j += kT) {
      const int t = generated[p.gen_offset + j];
      if (t >= 0 && t < V) atomicOr(&bitmap[t >> 5], 1u << (t & 31));
    }
    __syncthreads();
  }
  // x = logits / T, repetition penalty; the first maximum
  double bv = -INFINITY;
  int bi = -1;
  for (int base = tid; base < V; base += kB * kT) {
    float lv[kB];
#pragma unroll
    for (int j = 0; j < kB; ++j) lv[j] = base + j * kT < V ? lg[base + j * kT] : 0.0f;
#pragma unroll
    for (int j = 0; j < kB; ++j) {
      const int i = base + j * kT;
      if (i >= V) break;
      double v = static_cast<double>(lv[j]) / p.temperature;
      if (pen && ((bitmap[i >> 5] >> (i & 31)) & 1u))
        v = v > 0.0 ? v / p.repetition_penalty : v * p.repetition_penalty;
      X[i] = v;
      if (bi < 0 || v > bv) { bv = v; bi = i; }
    }
  }
  double m;
  int amax;
  block_argmax(bv, bi, sm, m, amax);   // its barriers also publish X

  uint64_t kkey = 0;
  if (p.top_k > 0 && p.top_k < V) kkey = kth_key(X, V, static_cast<uint32_t>(p.top_k), sm, cand);

  const bool topp = p.top_p < 1.0;
  uint64_t t_ge = 0, t_tie = 0;
  uint32_t r_ties = 0;
  if (topp) {
    double s = 0.0;
    for (int base = tid; base < V; base += kB * kT) {
      double xv[kB];
#pragma unroll
      for (int j = 0; j < kB; ++j) xv[j] = base + j * kT < V ? X[base + j * kT] : 0.0;
#pragma unroll
      for (int j = 0; j < kB; ++j) {
        const int i = base + j * kT;
        if (i >= V) break;
        const double e = okey(xv[j]) >= kkey ? exp(xv[j] - m) : 0.0;
        E[i] = e;
        s += e;
      }
    }
    const double S = block_sum(s, sm);   // barriers publish E
    top_p_bound(X, E, V, S, p.top_p, m, sm, cand);
    t_ge = sm.t_ge;
    t_tie = sm.t_tie;
    r_ties = sm.r_ties;
  }

  // the draw: warp w owns [w * seg, (w + 1) * seg)
  const int seg = ((V + kW - 1) / kW + 31) & ~31;
  const int lo = w * seg, hi = min(V, lo + seg);
  // kB chunks of 32 consecutive elements per batch, loads first
  double xv[kB], ev[kB];
  auto load = [&](int b0) {
#pragma unroll
    for (int j = 0; j < kB; ++j) {
      const int i = b0 + j * 32 + lane;
      xv[j] = i < hi ? X[i] : 0.0;
      ev[j] = (topp && i < hi) ? E[i] : 0.0;
    }
  };
  if (topp && r_ties) {
    uint32_t c = 0;
    for (int b0 = lo; b0 < hi; b0 += kB * 32) {
      load(b0);
#pragma unroll
      for (int j = 0; j < kB; ++j) {
        const bool tie = b0 + j * 32 + lane < hi && okey(xv[j]) == t_tie;
        c += __popc(__ballot_sync(0xffffffffu, tie));
      }
    }
    if (lane == 0) sm.tie_cnt[w] = c;
    __syncthreads();
    if (tid == 0) {
      uint32_t acc = 0;
      for (int k = 0; k < kW; ++k) { sm.tie_base[k] = acc; acc += sm.tie_cnt[k]; }
    }
    __syncthreads();
  }
  // the kept mass of element i (ties ranked in index order across the warp)
  auto mass = [&](int i, double x, double e_topp, uint32_t &ties) -> double {
    const bool valid = i < hi;
    const uint64_t key = okey(x);
    const bool tie = valid && topp && r_ties && key == t_tie;
    const unsigned bal = __ballot_sync(0xffffffffu, tie);
    const uint32_t rank = ties + __popc(bal & ((1u << lane) - 1u));
    ties += __popc(bal);
    double e = 0.0;
    if (valid) {
      const bool keep = !topp || key >= t_ge || (tie && rank < r_ties) || i == amax;
      if (keep) e = topp ? e_topp : (key >= kkey ? exp(x - m) : 0.0);
    }
    return e;
  };
  {
    uint32_t ties = (topp && r_ties) ? sm.tie_base[w] : 0u;
    double s = 0.0;
    for (int b0 = lo; b0 < hi; b0 += kB * 32) {
      load(b0);
#pragma unroll
      for (int j = 0; j < kB; ++j) s += mass(b0 + j * 32 + lane, xv[j], ev[j], ties);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) sm.seg[w] = s;
  }
  __syncthreads();
  if (tid == 0) {
    double tot = 0.0;
    for (int k = 0; k < kW; ++k) tot += sm.seg[k];
    const double target = p.u * tot;
    double acc = 0.0;
    int pw = -1, last = -1;
    for (int k = 0; k < kW; ++k) {
      if (sm.seg[k] > 0.0) last = k;
      if (pw < 0 && sm.seg[k] > 0.0 && acc + sm.seg[k] > target) { pw = k; break; }
      acc += sm.seg[k];
    }
    if (pw < 0) {   // u * total at the very end (rounding): the last segment with mass
      pw = last;
      acc = 0.0;
      for (int k = 0; k < last; ++k) acc += sm.seg[k];
    }
    if (pw < 0) out[r] = amax;   // no mass at all (non-finite logits)
    sm.pick_warp = pw;
    sm.pick_base = acc;
    sm.total = target;
  }
  __syncthreads();
  if (w == sm.pick_warp) {
    uint32_t ties = (topp && r_ties) ? sm.tie_base[w] : 0u;
    double base = sm.pick_base;
    const double target = sm.total;
    int pick = -1, last = -1;
    for (int b0 = lo; b0 < hi && pick < 0; b0 += kB * 32) {
      load(b0);
#pragma unroll
      for (int j = 0; j < kB; ++j) {
        const int i0 = b0 + j * 32;
        if (pick >= 0 || i0 >= hi) break;
        const double e = mass(i0 + lane, xv[j], ev[j], ties);
        double inc = e;   // inclusive scan in index order
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const double t = __shfl_up_sync(0xffffffffu, inc, o);
          if (lane >= o) inc += t;
        }
        const unsigned hit = __ballot_sync(0xffffffffu, e > 0.0 && base + inc > target);
        const unsigned pos = __ballot_sync(0xffffffffu, e > 0.0);
        if (hit) pick = i0 + __ffs(hit) - 1;
        else if (pos) last = i0 + 31 - __clz(pos);
        base += __shfl_sync(0xffffffffu, inc, 31);
      }
    }
    if (lane == 0) out[r] = pick >= 0 ? pick : (last >= 0 ? last : amax);
  }
}

}  // namespace

extern "C" size_t q3_sample_workspace_bytes(uint32_t rows, uint32_t vocab) {
  return 2 * sizeof(double) * static_cast<size_t>(rows) * vocab;
}

extern "C" int q3_sample_logits(const q3_view *logits, const q3_sample_row *params,
                                const int32_t *generated, int32_t *out_ids, void *workspace,
                                size_t workspace_bytes, void *stream) {
  if (!logits || !params || !out_ids || !logits->data) return Q3_ERR_NULL;
  if (logits->dtype != Q3_DT_F32) return Q3_ERR_DTYPE;
  const q3_view &l = *logits;
  if (l.rows == 0) return Q3_OK;
  if (l.cols == 0 || l.cols > (1u << 20) || l.col_bytes != 4 || l.row_bytes % 4 ||
      l.row_bytes < static_cast<int32_t>(4 * l.cols) || l.rows > 65535)
    return Q3_ERR_SHAPE;
  if (workspace_bytes < q3_sample_workspace_bytes(l.rows, l.cols) || !workspace) return Q3_ERR_CAPACITY;
  const size_t smem = 4 * (((l.cols + 31) / 32 + 1) & ~1u) + 16 * static_cast<size_t>(kCap);
  if (smem > 200 * 1024) return Q3_ERR_SHAPE;
  // per device (the attribute belongs to the current device's context)
  const cudaError_t e = cudaFuncSetAttribute(k_sample_rows, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(smem));
  if (e != cudaSuccess) { q3h::set_cuda_error(e); return Q3_ERR_CUDA; }
  k_sample_rows<<<l.rows, kT, smem, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const float *>(l.data), l.row_bytes / 4, static_cast<int>(l.cols), params, generated,
      out_ids, static_cast<double *>(workspace));
  return q3h::launch_status();
}

extern "C" int q3_rng_uniforms(uint64_t seed, uint32_t n, double *out) {
  if (!out && n) return Q3_ERR_NULL;
  q3rng::Pcg64 g(seed);
  for (uint32_t i = 0; i < n; ++i) out[i] = g.random();
  return Q3_OK;
}
