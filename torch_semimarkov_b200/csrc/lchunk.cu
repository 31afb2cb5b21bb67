// lchunk.cu -- time chunking of the float64 chains: plan, boundary check and
// offset fix-up.
//
// A chain is a linear recurrence in the linear domain: the values after a
// position are a positive linear function of the source window of its last
// K-1 positions.  Chunk j > 0 of a chain starts `warm` positions before its
// first output position from a uniform state; at the boundary jL its source
// window is compared with the window that chunk j-1 reached there.  Positive
// linear maps do not increase the Hilbert projective distance
//     d = max_i (l_e[i] - l_g[i]) - min_i (l_e[i] - l_g[i])     (log sources)
// so when d <= tol every later value of chunk j differs from the exact one by
// the same factor, exp(r), to relative error d.  The chunk's offsets
// D_j = D_{j-1} + r_j are added to its normalisers (n_tab) and to log Z.  A
// sequence with any boundary above tol is flagged; when the plan has a second
// warm-up its chunks are rerun with it and checked again, and a sequence that
// still does not join is rerun as one chain, so the result never rests on
// the guess.

#include "semicrf_internal.cuh"

namespace semicrf {

namespace {

constexpr int kLP = 8;           // positions per block of lchain_ws
constexpr double kTol = 1e-10;   // accepted projective distance at a boundary
constexpr double kNegl = 600.0;  // log sources this far below the window's max are negligible

__device__ __forceinline__ int seq_len(const int64_t* lengths, int b, int T) {
  const long long l = lengths[b];
  return l < 0 ? 0 : (l > T ? T : (int)l);
}

// one CTA per (boundary j, sequence, chain): r_j and whether it is acceptable.
// The two windows are read once into registers (KVP values per thread and
// window, for windows up to kVT * kVP entries; longer ones are read twice).
constexpr int kVT = 512, kVP = 16;

__device__ __forceinline__ double block_max(double v, double* sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int o = 16; o > 0; o >>= 1) v = fmax(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if (lane == 0) sh[warp] = v;
  __syncthreads();
  v = sh[0];
  for (int w = 1; w < kVT / 32; ++w) v = fmax(v, sh[w]);
  return v;
}

__global__ void __launch_bounds__(kVT) chunk_verify_kernel(const ChunkFix f0, const ChunkFix f1,
                                                           int kcap) {
  const ChunkFix& f = blockIdx.z ? f1 : f0;
  const int j = blockIdx.x + 1, b = blockIdx.y;
  if (f.only && !f.only[b]) return;
  const int nch = f.cp.nchunk;
  const int Lb = seq_len(f.lengths, b, f.T);
  __shared__ double s_a[kVT / 32], s_b[kVT / 32];
  if (j * f.cp.len >= Lb) {
    if (threadIdx.x == 0) {
      f.rdiff[(size_t)b * nch + j] = 0.0;
      f.okf[(size_t)b * nch + j] = 1;
    }
    return;
  }
  const int n = kcap * f.C;
  const double* e = f.hand + (((size_t)b * nch + (j - 1)) * 2 + 1) * (size_t)n;  // end of chunk j-1
  const double* g = f.hand + (((size_t)b * nch + j) * 2 + 0) * (size_t)n;        // guess of chunk j
  const bool cached = n <= kVT * kVP;
  double ev[kVP], gv[kVP];
  double me = -INFINITY, mg = -INFINITY;
  if (cached) {
#pragma unroll
    for (int r = 0; r < kVP; ++r) {
      const int i = threadIdx.x + r * kVT;
      ev[r] = i < n ? e[i] : -INFINITY;
      gv[r] = i < n ? g[i] : -INFINITY;
      me = fmax(me, ev[r]);
      mg = fmax(mg, gv[r]);
    }
  } else {
    for (int i = threadIdx.x; i < n; i += kVT) {
      me = fmax(me, e[i]);
      mg = fmax(mg, g[i]);
    }
  }
  // the largest log source of each window
  me = block_max(me, s_a);
  mg = block_max(mg, s_b);
  // spread of the differences over the entries that matter
  double dmin = INFINITY, dmax = -INFINITY;
  int bad = 0;
  auto take = [&](double x, double y) {
    const bool re = x > me - kNegl, rg = y > mg - kNegl;
    if (!re && !rg) return;
    if (!(x > -INFINITY) || !(y > -INFINITY)) {
      bad = 1;
      return;
    }
    const double d = x - y;
    dmin = fmin(dmin, d);
    dmax = fmax(dmax, d);
  };
  if (cached) {
#pragma unroll
    for (int r = 0; r < kVP; ++r)
      if (threadIdx.x + r * kVT < n) take(ev[r], gv[r]);
  } else {
    for (int i = threadIdx.x; i < n; i += kVT) take(e[i], g[i]);
  }
  dmax = block_max(dmax, s_a);
  dmin = -block_max(-dmin, s_b);
  bad = __syncthreads_or(bad);
  if (threadIdx.x == 0) {
    const bool ok = !bad && dmax >= dmin && (dmax - dmin) <= kTol;
    f.rdiff[(size_t)b * nch + j] = ok ? 0.5 * (dmax + dmin) : 0.0;
    f.okf[(size_t)b * nch + j] = ok ? 1 : 0;
  }
}

// per sequence: prefix sum of the offsets and the failure flag
__global__ void chunk_prefix_kernel(const ChunkFix f0, const ChunkFix f1) {
  const int bb = blockIdx.x * blockDim.x + threadIdx.x;
  if (bb >= 2 * f0.B) return;
  const ChunkFix& f = bb >= f0.B ? f1 : f0;
  const int b = bb >= f0.B ? bb - f0.B : bb;
  if (f.only && !f.only[b]) return;
  const int nch = f.cp.nchunk;
  const int Lb = seq_len(f.lengths, b, f.T);
  double acc = 0.0;
  int fail = 0;
  f.D[(size_t)b * nch] = 0.0;
  for (int j = 1; j < nch; ++j) {
    if (j * f.cp.len < Lb) {
      acc += f.rdiff[(size_t)b * nch + j];
      fail |= !f.okf[(size_t)b * nch + j];
    }
    f.D[(size_t)b * nch + j] = acc;
  }
  f.fail[b] = fail;
}

// add each chunk's offset to its normalisers (and log Z)
__global__ void chunk_apply_kernel(const ChunkFix f0, const ChunkFix f1) {
  const ChunkFix& f = blockIdx.y ? f1 : f0;
  const int nch = f.cp.nchunk, L = f.cp.len;
  const size_t total = (size_t)f.B * (f.T + 1);
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const int b = (int)(i / (f.T + 1)), t = (int)(i % (f.T + 1));
    if (f.fail[b] || (f.only && !f.only[b])) continue;
    const int Lb = seq_len(f.lengths, b, f.T);
    if (t > Lb) continue;
    const int u = f.dir == 0 ? t : Lb - t;
    int j = u <= L ? 0 : (u - 1) / L;
    if (j > nch - 1) j = nch - 1;
    if (f.n_tab && j > 0) f.n_tab[i] += f.D[(size_t)b * nch + j];
    if (t == 0 && f.dir == 0 && f.logz && Lb > 0) {
      int je = Lb <= L ? 0 : (Lb - 1) / L;
      if (je > nch - 1) je = nch - 1;
      const double lz = f.logz[b] + f.D[(size_t)b * nch + je];
      f.logz[b] = lz;
      if (f.partition) f.partition[b] = (float)lz;
    }
  }
}

}  // namespace

ChunkPlan chunk_plan(int B, int T, int K, int C, int nroles, int warm_override) {
  ChunkPlan p{1, T > 0 ? T : 1, 0, 0};
  if (B <= 0 || T <= 0 || warm_override < 0) return p;
  const int kcap = K > 1 ? K - 1 : 1;
  auto blocks = [](int w) { return ((w + kLP - 1) / kLP) * kLP; };
  const int sms = device_sm_count();
  // chunks for a given warm-up: as many as idle SMs allow, each at least
  // twice the warm-up long
  auto count = [&](int w) {
    int n = sms / (B * nroles);
    const int by_len = T / (2 * w);
    if (warm_override > 0 && n < 2) n = 2;
    return n > by_len ? by_len : n;
  };
  // Two warm-ups: the long one, twice the longest duration plus 64, and the
  // short one, the longest duration (the hand-off window must lie inside the
  // warm-up) plus 32.  How fast the window forgets the uniform start depends
  // on the scores; on configuration 2 (K = 300) every boundary joins after
  // K - 1 + 5 positions, on configuration 3 (K = 1000) not after K - 1 + 32.
  // When the long warm-up costs at most a quarter of the chunk length it
  // allows, it is the only one; otherwise the chunks run with the short one
  // and a sequence whose boundaries do not join reruns its chunks with the
  // long one.  warm_override > 0 gives the first warm-up in bits 0..15 and an
  // optional second one in bits 16..30.
  const int wl = blocks(2 * kcap + 64);
  int warm, warm2;
  if (warm_override > 0) {
    warm = warm_override & 0xffff;
    warm2 = (warm_override >> 16) & 0x7fff;
  } else {
    const int nl = count(wl);
    const int len_l = nl >= 2 ? blocks((T + nl - 1) / nl) : 0;
    if (nl >= 2 && 4 * wl <= len_l) {
      warm = wl;
      warm2 = 0;
    } else {
      warm = kcap + 32;
      warm2 = wl;
    }
  }
  if (warm < kcap) warm = kcap;  // the hand-off window must lie in the warm-up
  warm = blocks(warm);
  int nch = count(warm);
  if (nch < 2) return p;
  int len = (T + nch - 1) / nch;
  len = blocks(len);
  if (len < kcap) return p;
  p.nchunk = (T + len - 1) / len;
  if (p.nchunk < 2) return ChunkPlan{1, T, 0, 0};
  p.len = len;
  p.warm = warm;
  // the second warm-up must start at or after position 0 (u_out >= len)
  if (warm2 > 0) {
    warm2 = blocks(warm2 < kcap ? kcap : warm2);
    if (warm2 > len) warm2 = len;
    p.warm2 = warm2 > warm ? warm2 : 0;
  }
  return p;
}

size_t chunk_hand_doubles(int B, int K, int C, const ChunkPlan& cp) {
  const int kcap = K > 1 ? K - 1 : 1;
  return cp.nchunk > 1 ? (size_t)B * cp.nchunk * 2 * kcap * C : 0;
}

cudaError_t launch_chunk_fix(const ChunkFix& f0, const ChunkFix& f1, cudaStream_t s) {
  if (f0.B <= 0 || f0.cp.nchunk < 2) return cudaSuccess;
  const int kcap = f0.K > 1 ? f0.K - 1 : 1;
  chunk_verify_kernel<<<dim3(f0.cp.nchunk - 1, f0.B, 2), kVT, 0, s>>>(f0, f1, kcap);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  chunk_prefix_kernel<<<(2 * f0.B + 127) / 128, 128, 0, s>>>(f0, f1);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const size_t total = (size_t)f0.B * (f0.T + 1);
  int g = (int)((total + 255) / 256);
  if (g > device_sm_count() * 4) g = device_sm_count() * 4;
  chunk_apply_kernel<<<dim3(g, 2), 256, 0, s>>>(f0, f1);
  return cudaGetLastError();
}

}  // namespace semicrf
