// Sampling head over bf16 logits: repetition / presence penalty, temperature,
// top-k and top-p with injected uniforms, or greedy argmax.  One cluster of 8
// CTAs of 1024 threads per batch row, each CTA over one eighth of the
// vocabulary; the row's logits are re-read from L2 by each pass, and the
// CTAs' partial results (max, exp sums, radix histograms, candidates) meet in
// distributed shared memory at cluster barriers.
//
// Canonical rule (restated by oracle/rec_oracle.c:orc_sample):
//   x_i   = float(logit_i); for ids in the row's history: x = x<0 ? x*rho : x/rho
//           (rho != 1; mlx-lm repetition-penalty processor), then x -= alpha
//           (alpha != 0; the reference's presence mask, masked_sampling.py:99-100);
//           -0 is canonicalised to +0.
//   T = 0 : argmax x, lowest index among equal maxima (engine.py:284-285).
//   lse   = M + log(S), M = max x, S = sum exp(x - M) in this order: the ids
//           are cut into 8 chunks of Q = ceil(V / 8192) * 1024; in chunk c,
//           thread t sums ids cQ + t, cQ + t + 1024, ... in order, then a warp
//           butterfly, then the 32 warp sums in order; S = the 8 chunk sums in
//           order.  lp_i = x_i - lse.
//   (T, top_p, top_k) = (1, 1, 0): id = argmax(x_i + g_i)      (sampling.py:48-52)
//   top_k = 0 (top_p = 1): id = argmax(lp_i * (1/T) + g_i)     (mlx-lm categorical)
//   top_k > 0: the reference's joint filter (filtered_sampling.py:7-22) over the
//           stable ascending order of (x, index): theta = k-th largest x,
//           greater = #(x > theta); U_j = sum of exp(lp) of every element after j
//           in that order, accumulated in fp32 from the top; keep_p(j) <=> U_j <
//           top_p (the exact-arithmetic form of cumsum_j > 1 - top_p; always true
//           when top_p >= 1); keep = keep_p and (x > theta, or x == theta and
//           among the first (top_k - greater) tied elements, by index, from the
//           lowest-index tied element with keep_p).  id = argmax over kept of
//           lp * (1/T) + g, lowest index on ties.
//   g_i   = -log(-log(u_i)) with the injected uniform u_i (the reference draws it
//           with mx.random.gumbel; fixing u makes the ids comparable).
//   grammar mask (optional): x_i = -inf for every id whose allow bit is clear,
//           after the penalties (the reference's handoff, masked_sampling.py:101-110);
//           top_k = min(top_k, #allowed); no allowed id, or no finite candidate,
//           gives -1.
#pragma once
#include "common.cuh"

namespace rec {

constexpr int kSampleThreads = 1024;
constexpr int kSampleMaxCand = 1024;  // elements >= the top-k threshold (ties included)
constexpr int kSampleMaxTopK = 256;
constexpr int kSampleMaxVocab = 262144;

struct SampleArgs {
  const uint16_t* logits;  // bf16 [B, stride]
  int64_t stride;
  int V;
  const int* history;      // int32 [B, n_hist] or null
  int n_hist;
  float temperature, top_p, rep, presence;
  int top_k;
  const float* uniforms;   // fp32 [B, V] (temperature > 0)
  const uint32_t* allow;   // optional grammar mask: bit (i & 31) of word i >> 5 of row b set = id i allowed
  int64_t allow_stride;    // words per row of allow
  int* ids;                // int32 [B]; -1: more than kSampleMaxCand ties at the threshold, no id
                           // allowed, or no finite candidate
  // feedback mode (batch 1, a decode packet on the device): when ctl is set,
  // the history length is read from *hist_len, and the sampled id becomes
  // the session's next token, is recorded for the packet (with the EOS stop)
  // and is appended to history (up to hist_cap ids)
  int* ctl;
  int* hist_len;
  int* hist_out;
  int hist_cap;
};

// The control-block slots of a decode packet (decode.cu's Ctrl).
constexpr int kCtlSlotToken = 1, kCtlSlotActive = 3, kCtlSlotProduced = 4, kCtlSlotStep = 5, kCtlSlotNEos = 6,
              kCtlSlotEos = 8, kCtlSlotRecorded = 16, kCtlMaxRecorded = 64;

// Row b's sampled id (one thread): the output, and in feedback mode the
// packet bookkeeping that the decode step leaves to the sampler.
__device__ __forceinline__ void sample_finish(const SampleArgs& a, int b, int id) {
  a.ids[b] = id;
  if (!a.ctl) return;
  int* ctl = a.ctl;
  const int step = ctl[kCtlSlotStep] - 1;  // the decode step already advanced it
  if (ctl[kCtlSlotActive]) {
    if (step >= 0 && step < kCtlMaxRecorded) ctl[kCtlSlotRecorded + step] = id;
    ctl[kCtlSlotProduced] += 1;
    for (int i = 0; i < ctl[kCtlSlotNEos]; ++i)
      if (ctl[kCtlSlotEos + i] == id) ctl[kCtlSlotActive] = 0;
  }
  ctl[kCtlSlotToken] = id < 0 ? 0 : id;
  if (id >= 0 && a.hist_len && *a.hist_len < a.hist_cap) {
    a.hist_out[*a.hist_len] = id;
    *a.hist_len += 1;
  }
}

// Order-preserving unsigned key of a non-NaN float (-0 must be canonicalised).
__device__ __forceinline__ uint32_t float_key(float x) {
  const uint32_t u = __float_as_uint(x);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ float gumbel(float u) { return -rlog(-rlog(u)); }

// Cluster of kSampleCluster CTAs per row; CTA r owns the ids
// [r Q, (r + 1) Q) with Q = ceil(V / (kSampleCluster * 1024)) * 1024, and
// thread t of it the ids r Q + t + 1024 j.  Partial results meet through
// distributed shared memory at cluster barriers (no global scratch).
constexpr int kSampleCluster = 8;
constexpr int kSampleChunkWords = kSampleMaxVocab / kSampleCluster / 32;  // history bitmap words per CTA

struct SampleSmem {
  float red_v[32];
  int red_i[32];
  unsigned hist[256];
  unsigned seen[kSampleChunkWords];  // history bitmap of this CTA's ids
  float cx[kSampleMaxCand];          // this CTA's candidates
  int ci[kSampleMaxCand];
  float gx[kSampleMaxCand];          // all candidates (CTA 0)
  int gi[kSampleMaxCand];
  float sx[kSampleMaxCand];
  int si[kSampleMaxCand];
  float sp[kSampleMaxCand];
  float slp[kSampleMaxCand];
  int n_cand;
  uint32_t prefix, mask;
  int rank, tied, keep_lo, keep_hi;
  float lse;
  float M;
  int Mi;
  // published to the cluster (read by the other CTAs after a cluster barrier)
  float pub_v[2];
  int pub_i[2];
  unsigned pub_hist[2][256];
  float pub_S;
  int pub_n;
};

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Address of `p` (this CTA's shared memory) in the shared memory of cluster CTA `rank`.
template <class T>
__device__ __forceinline__ const T* peer(const T* p, int rank) {
  uint64_t out;
  asm volatile("mapa.u64 %0, %1, %2;" : "=l"(out) : "l"(reinterpret_cast<uint64_t>(p)), "r"(rank));
  return reinterpret_cast<const T*>(out);
}
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Histogram increment aggregated over the warp's lanes with the same bucket
// (the top digits of nearby logits collide heavily).
__device__ __forceinline__ void hist_add(unsigned* h, unsigned bucket) {
  const unsigned grp = __match_any_sync(__activemask(), bucket);
  if (int(threadIdx.x & 31) == __ffs(grp) - 1) atomicAdd(&h[bucket], unsigned(__popc(grp)));
}

// Block-wide argmax (value desc, index asc) of one value per thread; all
// threads return the result.
__device__ __forceinline__ void block_argmax(float& v, int& i, SampleSmem& s) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, off);
    const int oi = __shfl_xor_sync(0xffffffffu, i, off);
    if (ov > v || (ov == v && oi < i)) { v = ov; i = oi; }
  }
  if (lane == 0) { s.red_v[warp] = v; s.red_i[warp] = i; }
  __syncthreads();
  if (threadIdx.x == 0) {
    float bv = s.red_v[0];
    int bi = s.red_i[0];
    for (int w = 1; w < 32; ++w)
      if (s.red_v[w] > bv || (s.red_v[w] == bv && s.red_i[w] < bi)) { bv = s.red_v[w]; bi = s.red_i[w]; }
    s.M = bv;
    s.Mi = bi;
  }
  __syncthreads();
  v = s.M;
  i = s.Mi;
  __syncthreads();
}

// (value desc, index asc) arg-max over the cluster's published pub_v[k],
// pub_i[k] (after a cluster barrier); thread 0 writes s.M / s.Mi.
__device__ __forceinline__ void cluster_argmax(SampleSmem& s, int k) {
  if (threadIdx.x == 0) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int r = 0; r < kSampleCluster; ++r) {
      const float v = *peer(&s.pub_v[k], r);
      const int i = *peer(&s.pub_i[k], r);
      if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
    }
    s.M = bv;
    s.Mi = bi;
  }
  __syncthreads();
}

static __global__ void __cluster_dims__(kSampleCluster, 1, 1) __launch_bounds__(kSampleThreads, 1)
    k_sample(const SampleArgs a) {
  __shared__ SampleSmem s;
  extern __shared__ float xs[];  // x of this CTA's ids (pass 1 fills it; later passes read it)
  const int crank = int(cluster_rank());
  const int b = blockIdx.x / kSampleCluster, t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int V = a.V;
  const int Q = (V + kSampleCluster * kSampleThreads - 1) / (kSampleCluster * kSampleThreads) * kSampleThreads;
  const int lo = min(V, crank * Q), hi = min(V, lo + Q);
  const uint16_t* lg = a.logits + size_t(b) * a.stride;
  const bool pen = a.rep != 1.0f || a.presence != 0.0f;
  const int n_hist = a.hist_len ? *a.hist_len : a.n_hist;
  const uint32_t* allow = a.allow ? a.allow + size_t(b) * a.allow_stride : nullptr;
  const bool lead = crank == 0;
  if (pen) {
    for (int i = t; i < kSampleChunkWords; i += kSampleThreads) s.seen[i] = 0u;
    __syncthreads();
    for (int i = t; i < n_hist; i += kSampleThreads) {
      const int id = a.history[size_t(b) * n_hist + i];
      if (id >= lo && id < hi) atomicOr(&s.seen[(id - lo) >> 5], 1u << ((id - lo) & 31));
    }
    __syncthreads();
  }
  auto X = [&](int i) -> float {
    if (allow && !((allow[i >> 5] >> (i & 31)) & 1u)) return -INFINITY;  // grammar: not allowed
    float x = bf(lg[i]);
    if (pen && ((s.seen[(i - lo) >> 5] >> ((i - lo) & 31)) & 1u)) {
      if (a.rep != 1.0f) x = x < 0.0f ? __fmul_rn(x, a.rep) : __fdiv_rn(x, a.rep);
      if (a.presence != 0.0f) x = __fsub_rn(x, a.presence);
    }
    return __fadd_rn(x, 0.0f);
  };
  // with a grammar mask, top-k counts the allowed ids only
  int top_k = a.top_k;
  if (allow) {
    int c = 0;
    for (int w = (lo >> 5) + t; w < ((hi + 31) >> 5); w += kSampleThreads) {
      uint32_t m = allow[w];
      const int w0 = w << 5;
      if (w0 < lo) m &= ~0u << (lo - w0);
      if (w0 + 32 > hi) m &= (hi - w0 >= 32) ? ~0u : ((1u << (hi - w0)) - 1u);
      c += __popc(m);
    }
    c = __reduce_add_sync(0xffffffffu, c);
    if (lane == 0) s.red_i[warp] = c;
    __syncthreads();
    if (t == 0) {
      int n = 0;
      for (int w = 0; w < kSampleThreads / 32; ++w) n += s.red_i[w];
      s.pub_n = n;
    }
    cluster_sync_all();
    if (t == 0) {
      int n = 0;
      for (int r = 0; r < kSampleCluster; ++r) n += *peer(&s.pub_n, r);
      s.n_cand = n;
    }
    __syncthreads();
    const int n_allowed = s.n_cand;
    cluster_sync_all();  // every CTA has read pub_n
    if (n_allowed == 0) {
      if (lead && t == 0) sample_finish(a, b, -1);
      return;
    }
    top_k = top_k < n_allowed ? top_k : n_allowed;
  }
  const bool filtered = a.temperature != 0.0f && top_k > 0;

  // ---- pass 1: max (argmax for greedy) and the top digit's histogram
  if (filtered) {
    for (int i = t; i < 256; i += kSampleThreads) s.hist[i] = 0u;
    __syncthreads();
  }
  float mx = -INFINITY;
  int mi = 0x7fffffff;
#pragma unroll 4
  for (int i = lo + t; i < hi; i += kSampleThreads) {
    const float x = X(i);
    xs[i - lo] = x;
    if (x > mx) { mx = x; mi = i; }
    if (filtered) hist_add(s.hist, float_key(x) >> 24);
  }
  block_argmax(mx, mi, s);
  if (t == 0) {
    s.pub_v[0] = mx;
    s.pub_i[0] = mi;
  }
  if (filtered)
    for (int i = t; i < 256; i += kSampleThreads) s.pub_hist[0][i] = s.hist[i];
  cluster_sync_all();
  cluster_argmax(s, 0);
  // cluster-wide histogram of a level from pub_hist[p]
  auto gather_hist = [&](int p) {
    for (int i = t; i < 256; i += kSampleThreads) {
      unsigned c = 0;
      for (int r = 0; r < kSampleCluster; ++r) c += *peer(&s.pub_hist[p][i], r);
      s.hist[i] = c;
    }
    __syncthreads();
  };
  if (filtered) gather_hist(0);
  const float M = s.M;
  if (a.temperature == 0.0f) {  // no finite candidate (all masked or -inf): -1
    if (lead && t == 0) sample_finish(a, b, s.Mi == 0x7fffffff ? -1 : s.Mi);
    cluster_sync_all();  // the peers' published values stay readable until every CTA is done
    return;
  }

  // radix select of the k-th largest key: resolve one digit from s.hist
  auto resolve = [&](int level) {
    if (t == 0) {
      const int shift = 24 - 8 * level;
      int rank = level == 0 ? top_k - 1 : s.rank;
      unsigned c = 0;
      int d = 255;
      for (; d > 0; --d) {
        if (c + s.hist[d] > unsigned(rank)) break;
        c += s.hist[d];
      }
      s.rank = rank - int(c);
      s.prefix = (level == 0 ? 0u : s.prefix) | (uint32_t(d) << shift);
      s.mask = (level == 0 ? 0u : s.mask) | (0xFFu << shift);
      if (level == 3) s.tied = int(s.hist[d]);
    }
    __syncthreads();
  };
  auto local_hist = [&](int level) {  // this CTA's elements matching the prefix of levels < level
    for (int i = t; i < 256; i += kSampleThreads) s.hist[i] = 0u;
    __syncthreads();
    const uint32_t pre = s.prefix, msk = s.mask;
    const int shift = 24 - 8 * level;
    for (int i = t; i < hi - lo; i += kSampleThreads) {
      const uint32_t k = float_key(xs[i]);
      if ((k & msk) == pre) hist_add(s.hist, (k >> shift) & 255u);
    }
    __syncthreads();
  };
  if (filtered) resolve(0);

  // ---- pass 2: this CTA's share of S (canonical order) [+ next digit]
  {
    float sum = 0.0f;
    for (int i = t; i < hi - lo; i += kSampleThreads) sum = __fadd_rn(sum, rexp(__fsub_rn(xs[i], M)));
    sum = bfly_sum(sum);
    if (lane == 0) s.red_v[warp] = sum;
    __syncthreads();
    if (t == 0) {
      float tot = 0.0f;
      for (int w = 0; w < 32; ++w) tot = __fadd_rn(tot, s.red_v[w]);
      s.pub_S = tot;
    }
    if (filtered) {
      local_hist(1);
      for (int i = t; i < 256; i += kSampleThreads) s.pub_hist[1][i] = s.hist[i];
    }
    cluster_sync_all();
    if (t == 0) {
      float tot = 0.0f;  // S = the CTAs' shares in cluster order
      for (int r = 0; r < kSampleCluster; ++r) tot = __fadd_rn(tot, *peer(&s.pub_S, r));
      s.lse = __fadd_rn(M, rlog(tot));
    }
    __syncthreads();
    if (filtered) {
      gather_hist(1);
      resolve(1);
    }
  }
  const float lse = s.lse;
  const float inv_t = __fdiv_rn(1.0f, a.temperature);
  const float* u = a.uniforms + size_t(b) * V;

  if (!filtered) {
    const bool t1 = a.temperature == 1.0f && a.top_p >= 1.0f;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll 4
    for (int i = lo + t; i < hi; i += kSampleThreads) {
      const float x = xs[i - lo];
      const float z = t1 ? __fadd_rn(x, gumbel(u[i])) : __fadd_rn(__fmul_rn(__fsub_rn(x, lse), inv_t), gumbel(u[i]));
      if (z > bv) { bv = z; bi = i; }
    }
    block_argmax(bv, bi, s);
    if (t == 0) {
      s.pub_v[1] = bv;
      s.pub_i[1] = bi;
    }
    cluster_sync_all();
    cluster_argmax(s, 1);
    if (lead && t == 0) sample_finish(a, b, s.Mi == 0x7fffffff ? -1 : s.Mi);
    cluster_sync_all();
    return;
  }

  for (int level = 2; level < 4; ++level) {
    local_hist(level);
    for (int i = t; i < 256; i += kSampleThreads) s.pub_hist[level & 1][i] = s.hist[i];
    cluster_sync_all();
    gather_hist(level & 1);
    resolve(level);
  }
  const uint32_t theta = s.prefix;
  const int greater = top_k - 1 - s.rank;
  const int n = greater + s.tied;
  if (n > kSampleMaxCand) {
    if (lead && t == 0) sample_finish(a, b, -1);
    cluster_sync_all();
    return;
  }
  // ---- collect this CTA's elements >= theta, then CTA 0 gathers them
  if (t == 0) s.n_cand = 0;
  __syncthreads();
  for (int i = lo + t; i < hi; i += kSampleThreads) {
    const float x = xs[i - lo];
    if (float_key(x) >= theta) {
      const int slot = atomicAdd(&s.n_cand, 1);
      if (slot < kSampleMaxCand) {
        s.cx[slot] = x;
        s.ci[slot] = i;
      }
    }
  }
  __syncthreads();
  if (t == 0) s.pub_n = s.n_cand;
  cluster_sync_all();
  if (lead) {
    // CTA r's candidates go to [off_r, off_r + n_r); the order is irrelevant
    // (they are ranked by value and index below)
    int off = 0;
    for (int r = 0; r < kSampleCluster; ++r) {
      const int nr = *peer(&s.pub_n, r);
      for (int q = t; q < nr && off + q < kSampleMaxCand; q += kSampleThreads) {
        s.gx[off + q] = *peer(&s.cx[q], r);
        s.gi[off + q] = *peer(&s.ci[q], r);
      }
      off += nr;
    }
  }
  cluster_sync_all();  // the other CTAs may exit once CTA 0 has read their candidates
  if (!lead) return;
  __syncthreads();
  // descending (x desc, index desc) by rank counting
  if (t < n) {
    const float xi = s.gx[t];
    const int ii = s.gi[t];
    int r = 0;
    for (int j = 0; j < n; ++j) {
      const float xj = s.gx[j];
      const int ij = s.gi[j];
      r += (xj > xi || (xj == xi && ij > ii)) ? 1 : 0;
    }
    s.sx[r] = xi;
    s.si[r] = ii;
  }
  __syncthreads();
  if (t < n) {
    const float lp = __fsub_rn(s.sx[t], lse);
    s.slp[t] = lp;
    s.sp[t] = rexp(lp);
  }
  __syncthreads();
  if (t == 0) {
    // keep_p along the descending order; cx reused as flags
    const bool use_p = a.top_p < 1.0f;
    float U = 0.0f;
    for (int q = 0; q < n; ++q) {
      s.cx[q] = (!use_p || U < a.top_p) ? 1.0f : 0.0f;
      U = __fadd_rn(U, s.sp[q]);
    }
    // tied elements occupy q in [greater, n), index descending; the lowest
    // index with keep_p is the largest such q
    int first = -1;
    for (int q = n - 1; q >= greater; --q)
      if (s.cx[q] != 0.0f) { first = q; break; }
    const int allowed = top_k - greater;
    s.keep_lo = first < 0 ? n : max(greater, first - allowed + 1);
    s.keep_hi = first;  // tied kept: q in [keep_lo, keep_hi]
  }
  __syncthreads();
  if (warp == 0) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int q = lane; q < n; q += 32) {
      const bool keep = q < greater ? (s.cx[q] != 0.0f) : (q >= s.keep_lo && q <= s.keep_hi);
      if (!keep) continue;
      const int i = s.si[q];
      const float z = __fadd_rn(__fmul_rn(s.slp[q], inv_t), gumbel(u[i]));
      if (z > bv || (z == bv && i < bi)) { bv = z; bi = i; }
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if (lane == 0) sample_finish(a, b, bi == 0x7fffffff ? -1 : bi);
  }
}

// B rows, one cluster of kSampleCluster CTAs each.
__host__ inline cudaError_t launch_sample(const SampleArgs& a, int batch, cudaStream_t st) {
  const int Q = (a.V + kSampleCluster * kSampleThreads - 1) / (kSampleCluster * kSampleThreads) * kSampleThreads;
  const size_t dyn = size_t(Q) * sizeof(float);
  cudaError_t e = cudaFuncSetAttribute(k_sample, cudaFuncAttributeMaxDynamicSharedMemorySize, int(dyn));
  if (e != cudaSuccess) return e;
  k_sample<<<batch * kSampleCluster, kSampleThreads, dyn, st>>>(a);
  return cudaGetLastError();
}

}  // namespace rec
