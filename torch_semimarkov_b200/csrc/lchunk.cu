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

// one CTA per (boundary j, sequence): r_j and whether it is acceptable
__global__ void __launch_bounds__(256) chunk_verify_kernel(const ChunkFix f, int kcap) {
  const int j = blockIdx.x + 1, b = blockIdx.y;
  if (f.only && !f.only[b]) return;
  const int nch = f.cp.nchunk;
  const int Lb = seq_len(f.lengths, b, f.T);
  __shared__ double s_mx[2][8], s_mn[8], s_mxd[8];
  __shared__ int s_bad[8];
  if (j * f.cp.len >= Lb) {
    if (threadIdx.x == 0) {
      f.rdiff[(size_t)b * nch + j] = 0.0;
      f.okf[(size_t)b * nch + j] = 1;
    }
    return;
  }
  const size_t n = (size_t)kcap * f.C;
  const double* e = f.hand + (((size_t)b * nch + (j - 1)) * 2 + 1) * n;  // end of chunk j-1
  const double* g = f.hand + (((size_t)b * nch + j) * 2 + 0) * n;        // guess of chunk j
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // pass 1: the largest log source of each window
  double me = -INFINITY, mg = -INFINITY;
  for (size_t i = threadIdx.x; i < n; i += blockDim.x) {
    me = fmax(me, e[i]);
    mg = fmax(mg, g[i]);
  }
  for (int o = 16; o > 0; o >>= 1) {
    me = fmax(me, __shfl_xor_sync(0xffffffffu, me, o));
    mg = fmax(mg, __shfl_xor_sync(0xffffffffu, mg, o));
  }
  if (lane == 0) {
    s_mx[0][warp] = me;
    s_mx[1][warp] = mg;
  }
  __syncthreads();
  me = s_mx[0][0];
  mg = s_mx[1][0];
  for (int w = 1; w < (int)(blockDim.x >> 5); ++w) {
    me = fmax(me, s_mx[0][w]);
    mg = fmax(mg, s_mx[1][w]);
  }
  // pass 2: spread of the differences over the entries that matter
  double dmin = INFINITY, dmax = -INFINITY;
  int bad = 0;
  for (size_t i = threadIdx.x; i < n; i += blockDim.x) {
    const double x = e[i], y = g[i];
    const bool re = x > me - kNegl, rg = y > mg - kNegl;
    if (!re && !rg) continue;
    if (!(x > -INFINITY) || !(y > -INFINITY)) {
      bad = 1;
      continue;
    }
    const double d = x - y;
    dmin = fmin(dmin, d);
    dmax = fmax(dmax, d);
  }
  for (int o = 16; o > 0; o >>= 1) {
    dmin = fmin(dmin, __shfl_xor_sync(0xffffffffu, dmin, o));
    dmax = fmax(dmax, __shfl_xor_sync(0xffffffffu, dmax, o));
    bad |= __shfl_xor_sync(0xffffffffu, bad, o);
  }
  if (lane == 0) {
    s_mn[warp] = dmin;
    s_mxd[warp] = dmax;
    s_bad[warp] = bad;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) {
      dmin = fmin(dmin, s_mn[w]);
      dmax = fmax(dmax, s_mxd[w]);
      bad |= s_bad[w];
    }
    if (s_mn[0] < dmin) dmin = s_mn[0];
    if (s_mxd[0] > dmax) dmax = s_mxd[0];
    bad |= s_bad[0];
    const bool ok = !bad && dmax >= dmin && (dmax - dmin) <= kTol;
    f.rdiff[(size_t)b * nch + j] = ok ? 0.5 * (dmax + dmin) : 0.0;
    f.okf[(size_t)b * nch + j] = ok ? 1 : 0;
  }
}

// per sequence: prefix sum of the offsets and the failure flag
__global__ void chunk_prefix_kernel(const ChunkFix f) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= f.B) return;
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
__global__ void chunk_apply_kernel(const ChunkFix f) {
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

cudaError_t launch_chunk_fix(const ChunkFix& f, cudaStream_t s) {
  if (f.B <= 0 || f.cp.nchunk < 2) return cudaSuccess;
  const int kcap = f.K > 1 ? f.K - 1 : 1;
  chunk_verify_kernel<<<dim3(f.cp.nchunk - 1, f.B), 256, 0, s>>>(f, kcap);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  chunk_prefix_kernel<<<(f.B + 127) / 128, 128, 0, s>>>(f);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const size_t total = (size_t)f.B * (f.T + 1);
  int g = (int)((total + 255) / 256);
  if (g > device_sm_count() * 8) g = device_sm_count() * 8;
  chunk_apply_kernel<<<g, 256, 0, s>>>(f);
  return cudaGetLastError();
}

}  // namespace semicrf
