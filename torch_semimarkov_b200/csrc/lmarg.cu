// lmarg.cu -- log-semiring gradients from the alpha and beta chain tables.
//
// The backward of the streaming scan (pytorch_reference.py:276-525, the
// marginals at :458-499) needs, per sequence b, the segment marginals
//     P(t -> t+k, c) = exp(A[t,c] + ps[t,c] - cum[t,c] + db[min(k,K-1),c]
//                          + cum[t+k,c] + pe[t+k-1,c] + beta[t+k,c] - logZ)
// where A[t,c] = LSE_c' (alpha[t,c'] + tr[c',c]) and beta[s,c] is the
// backward value of a segment ending at s with label c.  Both chains run
// before this file (lchain_ws.cu / lchain.cu) and leave float64 tables with a
// per-position normaliser n:
//     alpha chain:  xa = exp(alpha - xn),  xA = exp(A - xn)
//     beta  chain:  ya = exp(G - yn),      yA = exp(beta - yn)
// with G[t,c] = ps[t,c] + LSE_k(db + cum[t+k] - cum[t] + pe[t+k-1] + beta[t+k]).
// From these every gradient is a parallel map or reduction -- no serial
// dependency is left:
//   Pend[t,c]   = xa*yA*f_t,  Pstart[t,c] = xA*ya*f_t,  f_t = exp(xn+yn-logZ)
//   grad_cum[t] = g (Pend - Pstart), grad_ps[t] = g Pstart, grad_pe[t-1] = g Pend
//   grad_tr[c',c] = exp(tr[c',c]) sum_b g_b sum_t xa[t,c'] f_t ya[t,c]
//   grad_db[k,c]  = exp(db[k,c]) sum_b g_b sum_t X[t,c] Y[t+k,c]
// where X/Y split the segment marginal into a start and an end factor,
// re-referenced per tile of targets so that both stay inside float64 range.
// Partials are per (sequence, chunk) and summed in a fixed order: no atomics.

#include <cstdlib>
#include <cstring>

#include "semicrf_internal.cuh"

namespace semicrf {

namespace {

constexpr int kMT = 256;
constexpr int kTT = 64;  // positions per block (targets per correlation tile)
constexpr double kDbFlag = 600.0;  // block-factor exponent beyond which a sequence is redone

__device__ __forceinline__ int seq_len(const int64_t* lengths, int b, int T) {
  const long long l = lengths[b];
  return l < 0 ? 0 : (l > T ? T : (int)l);
}

// ---- per-position marginals and block-relative factors -----------------------
// One CTA per (64-position block, label group of at most kPG labels, sequence).
// Each element (t, c) of the block gives the marginals -> grad_cum /
// grad_ps / grad_pe and the start and end factors in the split form
//     exp(la) = xA exp(sa),  sa = xn + ps - cum   (t < len),
//     exp(lb) = yA exp(sb),  sb = yn + cum + pe   (t >= 1),
// which stay in shared memory; then per label a block reference maX / mbY and
// the linear factors xA exp(sa - maX), yA exp(sb - mbY) go to global memory.
// The reference only has to bound the block's log factors from above (every
// linear factor is then at most 1) and lie close to their maximum (so that the
// largest stays near 1): it is the maximum of (e + 1) ln 2 + s, e the binary
// exponent of xA or yA, which exceeds log xA + s by less than ln 2.  So no
// logarithm is taken, and f_t = exp(xn + yn - logZ) once per row: two
// exponentials per element instead of five transcendentals.  One pass over
// the tables: the factors are never written out and read back.
constexpr int kPG = 32;  // labels per CTA

// (e + 1) ln 2 + s >= log v + s for v > 0 with binary exponent e (a subnormal
// v counts as e = -1023, still a bound); -inf where the factor is absent
__device__ __forceinline__ double log_bound(double v, double s) {
  if (!(v > 0.0) || !(s > -INFINITY)) return -INFINITY;
  const int e = (int)((__double_as_longlong(v) >> 52) & 0x7ff) - 1023;
  return (double)(e + 1) * 0.69314718055994531 + s;
}

// v exp(s - mx) (at most 1: mx bounds log v + s); where exp(s - mx) alone
// would overflow (a tiny v near the block maximum) it is exp(log v + s - mx)
__device__ __forceinline__ double linear_factor(double v, double s, double mx) {
  if (!(v > 0.0) || !(s > -INFINITY)) return 0.0;
  const double d = s - mx;
  return d < 700.0 ? v * exp(d) : exp(log(v) + d);
}

__host__ __device__ inline int posblk_ld(int C) { return (C < kPG ? C : kPG) | 1; }
__host__ __device__ inline int posblk_smem(int C) { return 4 * kTT * posblk_ld(C) * 8; }

// W consecutive labels per item (W = 2: 16-byte table loads and stores, half
// the index work; the host picks it when C is even and every pointer is aligned)
template <int W>
__global__ void __launch_bounds__(kMT, 4) lmarg_posblk_kernel(const LMargArgs a) {
  extern __shared__ __align__(16) unsigned char pbsm[];
  __shared__ double srow[3][kTT];  // xn, yn, f_t of each row
  __shared__ double smx[2][kPG];
  const int C = a.C, T = a.T;
  const int blk = blockIdx.x, g0 = blockIdx.y * kPG, b = blockIdx.z;
  const int cgn = min(kPG, C - g0);
  const int ld = posblk_ld(C);  // odd: the column maxima read without bank conflicts
  double* sxA = reinterpret_cast<double*>(pbsm);  // [kTT][ld] xA (0: no start factor)
  double* ssa = sxA + kTT * ld;                  // [kTT][ld] sa
  double* syA = ssa + kTT * ld;                  // [kTT][ld] yA (0: no end factor)
  double* ssb = syA + kTT * ld;                  // [kTT][ld] sb
  const int t0 = blk * kTT, nt = min(kTT, T + 1 - t0);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int Lb = seq_len(a.lengths, b, T);
  const double g = (double)a.grad_output[b];
  const double lz = a.logz[b];
  const float* cum_b = a.cum + (size_t)b * (T + 1) * C;
  for (int ti = tid; ti < nt; ti += kMT) {
    const int t = t0 + ti;
    double xn = 0.0, yn = 0.0, f = 0.0;
    if (Lb >= 1 && t <= Lb) {
      const size_t row = (size_t)b * (T + 1) + t;
      xn = a.xn[row];
      yn = a.yn[row];
      f = exp(xn + yn - lz);
    }
    srow[0][ti] = xn;
    srow[1][ti] = yn;
    srow[2][ti] = f;
  }
  __syncthreads();
  // W-wide loads and stores of the tables (aligned: checked by the host)
  auto ldd = [](const double* p, double (&v)[W]) {
    if constexpr (W == 2) {
      const double2 q = *reinterpret_cast<const double2*>(p);
      v[0] = q.x;
      v[1] = q.y;
    } else {
      v[0] = *p;
    }
  };
  auto ldf = [](const float* p, double (&v)[W]) {
    if constexpr (W == 2) {
      const float2 q = *reinterpret_cast<const float2*>(p);
      v[0] = (double)q.x;
      v[1] = (double)q.y;
    } else {
      v[0] = (double)*p;
    }
  };
  auto stf = [](float* p, const float (&v)[W]) {
    if constexpr (W == 2) {
      *reinterpret_cast<float2*>(p) = make_float2(v[0], v[1]);
    } else {
      *p = v[0];
    }
  };
  auto std_ = [](double* p, const double (&v)[W]) {
    if constexpr (W == 2) {
      *reinterpret_cast<double2*>(p) = make_double2(v[0], v[1]);
    } else {
      *p = v[0];
    }
  };
  // kPB items (2 labels) per thread at a time, all their loads issued before
  // the first store (the stores could alias the tables as far as the compiler knows)
  constexpr int kPB = 2 / W;
  const int nw = cgn / W;  // items per row
  const int ne = nt * nw;
  // item e = (row e / nw, labels W * (e % nw) ..), stepped by kMT without divisions
  const int dq = kMT / nw, dr = kMT % nw;
  auto step = [&](int& ti, int& ci) {
    ti += dq;
    ci += dr;
    if (ci >= nw) {
      ci -= nw;
      ++ti;
    }
  };
  int ti0 = tid / nw, ci0 = tid % nw;
  for (int e0 = tid; e0 < ne; e0 += kPB * kMT) {
    // vsa = ps - cum, vsb = cum + pe
    double vxA[kPB][W], vyA[kPB][W], vxa[kPB][W], vya[kPB][W], vsa[kPB][W], vsb[kPB][W];
    int tis[kPB], cis[kPB];
#pragma unroll
    for (int j = 0; j < kPB; ++j) {
      const int e = e0 + j * kMT;
      tis[j] = ti0;
      cis[j] = ci0;
      step(ti0, ci0);
      const int t = t0 + tis[j], c = g0 + W * cis[j];
      const size_t i = ((size_t)b * (T + 1) + t) * C + c;
#pragma unroll
      for (int w = 0; w < W; ++w) vxA[j][w] = vyA[j][w] = vxa[j][w] = vya[j][w] = vsa[j][w] = vsb[j][w] = 0.0;
      if (e < ne && Lb >= 1 && t <= Lb) {
        ldd(a.xA + i, vxA[j]);
        ldd(a.yA + i, vyA[j]);
        if (t >= 1) ldd(a.xa + i, vxa[j]);
        if (t < Lb) ldd(a.ya + i, vya[j]);
        double cu[W], ps[W], pe[W];
        ldf(cum_b + (size_t)t * C + c, cu);
#pragma unroll
        for (int w = 0; w < W; ++w) ps[w] = pe[w] = 0.0;
        if (a.ps && t < Lb) ldf(a.ps + ((size_t)b * T + t) * C + c, ps);
        if (a.pe && t >= 1) ldf(a.pe + ((size_t)b * T + t - 1) * C + c, pe);
#pragma unroll
        for (int w = 0; w < W; ++w) {
          vsa[j][w] = ps[w] - cu[w];
          vsb[j][w] = cu[w] + pe[w];
        }
      }
    }
#pragma unroll
    for (int j = 0; j < kPB; ++j) {
      const int e = e0 + j * kMT;
      if (e >= ne) break;
      const int ti = tis[j], cc = W * cis[j];
      const int t = t0 + ti, c = g0 + cc;
      const size_t i = ((size_t)b * (T + 1) + t) * C + c;
      double pend[W], pst[W];
#pragma unroll
      for (int w = 0; w < W; ++w) {
        pend[w] = pst[w] = 0.0;
        double xv = 0.0, yv = 0.0, sa = 0.0, sb = 0.0;
        if (Lb >= 1 && t <= Lb) {
          const double f = srow[2][ti];
          if (t >= 1) pend[w] = vxa[j][w] * vyA[j][w] * f;
          if (t < Lb) {
            pst[w] = vxA[j][w] * vya[j][w] * f;
            xv = vxA[j][w];
            sa = srow[0][ti] + vsa[j][w];
          }
          if (t >= 1) {
            yv = vyA[j][w];
            sb = srow[1][ti] + vsb[j][w];
          }
        }
        sxA[ti * ld + cc + w] = xv;
        ssa[ti * ld + cc + w] = sa;
        syA[ti * ld + cc + w] = yv;
        ssb[ti * ld + cc + w] = sb;
      }
      float gv[W];
#pragma unroll
      for (int w = 0; w < W; ++w) gv[w] = (float)(g * (pend[w] - pst[w]));
      stf(a.grad_cum + i, gv);
      if (a.grad_ps && t < T) {
#pragma unroll
        for (int w = 0; w < W; ++w) gv[w] = (float)(g * pst[w]);
        stf(a.grad_ps + ((size_t)b * T + t) * C + c, gv);
      }
      if (a.grad_pe && t >= 1) {
#pragma unroll
        for (int w = 0; w < W; ++w) gv[w] = (float)(g * pend[w]);
        stf(a.grad_pe + ((size_t)b * T + t - 1) * C + c, gv);
      }
    }
  }
  __syncthreads();
  // block references: one warp per (label, table), two rows per lane
  for (int w = warp; w < 2 * cgn; w += kMT / 32) {
    const int cc = w >> 1;
    const bool isb = w & 1;
    const double* v = isb ? syA : sxA;
    const double* sv = isb ? ssb : ssa;
    double m = -INFINITY;
    for (int ti = lane; ti < nt; ti += 32) m = fmax(m, log_bound(v[ti * ld + cc], sv[ti * ld + cc]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmax(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) smx[isb][cc] = m;
  }
  __syncthreads();
  const int nblk = (T + 1 + kTT - 1) / kTT;
  ti0 = tid / nw;
  ci0 = tid % nw;
  for (int e = tid; e < ne; e += kMT, step(ti0, ci0)) {
    const int ti = ti0, cc = W * ci0;
    const size_t i = ((size_t)b * (T + 1) + t0 + ti) * C + g0 + cc;
    double xl[W], yl[W];
#pragma unroll
    for (int w = 0; w < W; ++w) {
      xl[w] = linear_factor(sxA[ti * ld + cc + w], ssa[ti * ld + cc + w], smx[0][cc + w]);
      yl[w] = linear_factor(syA[ti * ld + cc + w], ssb[ti * ld + cc + w], smx[1][cc + w]);
    }
    std_(a.la + i, xl);
    std_(a.lb + i, yl);
  }
  if (tid < cgn) {
    const size_t j = ((size_t)b * nblk + blk) * C + g0 + tid;
    a.maX[j] = smx[0][tid];
    a.mbY[j] = smx[1][tid];
  }
  if (blk == 0 && blockIdx.y == 0 && tid == 0) a.dbflag[b] = 0;  // lmarg_db_kernel sets it
}

// the paired kernel needs an even C and 16-byte (tables) / 8-byte (scores,
// gradients) aligned bases
bool posblk_pairs(const LMargArgs& a) {
  auto al = [](const void* p, uintptr_t n) { return p == nullptr || (uintptr_t)p % n == 0; };
  return a.C % 2 == 0 && al(a.xA, 16) && al(a.yA, 16) && al(a.xa, 16) && al(a.ya, 16) &&
         al(a.la, 16) && al(a.lb, 16) && al(a.cum, 8) && al(a.ps, 8) && al(a.pe, 8) &&
         al(a.grad_cum, 8) && al(a.grad_ps, 8) && al(a.grad_pe, 8);
}

// ---- transition partials for C <= 24: the same sums, with every thread busy ----
// 8x8 threads hold 3x3 tiles of the 24x24 pair block (9 FMAs per 6 shared-memory
// loads); the four 64-thread groups take every fourth staged position, and
// their partial tiles are added in group order at the end.  Positions are
// staged TS at a time; the next stage's table rows are loaded into registers
// while the current one computes, and f_t scales the x values as they are read.
__global__ void __launch_bounds__(kMT) lmarg_tr24_kernel(const LMargArgs a) {
  constexpr int PB = 24, TS = 96, NG = kMT / 64, NE = TS * PB / kMT;
  static_assert(TS * PB % kMT == 0, "whole stage per thread count");
  __shared__ __align__(16) double xs[TS][PB];
  __shared__ __align__(16) double ys[TS][PB];
  __shared__ double fs[TS];
  // the groups' partial tiles reuse the staging buffer once the loop is done
  static_assert((NG - 1) * 9 * 64 <= TS * PB, "partials fit in the x stage");
  double(*red)[9][64] = reinterpret_cast<double(*)[9][64]>(&xs[0][0]);
  const int C = a.C, T = a.T;
  const int ch = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, grp = tid >> 6, l = tid & 63, tx = l & 7, ty = l >> 3;
  const int Lb = seq_len(a.lengths, b, T);
  const int per = (T + a.nchunk - 1) / a.nchunk;
  const int t_lo = ch * per;
  const int t_hi = min(t_lo + per, Lb);
  double acc[3][3];
#pragma unroll
  for (int i = 0; i < 3; ++i)
#pragma unroll
    for (int j = 0; j < 3; ++j) acc[i][j] = 0.0;
  const double lz = a.logz[b];
  const size_t rowb = (size_t)b * (T + 1);
  double px[NE], py[NE], pf = 0.0;
  auto prefetch = [&](int t0) {
    const int n = min(TS, t_hi - t0);
#pragma unroll
    for (int r = 0; r < NE; ++r) {
      const int e = tid + r * kMT;
      const int i = e / PB, q = e % PB;
      px[r] = py[r] = 0.0;
      if (i < n && q < C) {
        const size_t row = (rowb + t0 + i) * C;
        px[r] = a.xa[row + q];
        py[r] = a.ya[row + q];
      }
    }
    pf = (tid < n) ? a.xn[rowb + t0 + tid] + a.yn[rowb + t0 + tid] : 0.0;
  };
  if (t_lo < t_hi) prefetch(t_lo);
  for (int t0 = t_lo; t0 < t_hi; t0 += TS) {
    const int n = min(TS, t_hi - t0);
    __syncthreads();  // the previous stage's reads are done
#pragma unroll
    for (int r = 0; r < NE; ++r) {
      const int e = tid + r * kMT;
      xs[e / PB][e % PB] = px[r];
      ys[e / PB][e % PB] = py[r];
    }
    if (tid < TS) fs[tid] = tid < n ? exp(pf - lz) : 0.0;
    __syncthreads();
    if (t0 + TS < t_hi) prefetch(t0 + TS);  // in flight during the FMAs below
    for (int i = grp; i < n; i += NG) {
      const double f = fs[i];
      double xv[3], yv[3];
#pragma unroll
      for (int q = 0; q < 3; ++q) {
        xv[q] = xs[i][ty * 3 + q] * f;
        yv[q] = ys[i][tx * 3 + q];
      }
#pragma unroll
      for (int p = 0; p < 3; ++p)
#pragma unroll
        for (int q = 0; q < 3; ++q) acc[p][q] = fma(xv[p], yv[q], acc[p][q]);
    }
  }
  __syncthreads();  // every read of the last stage is done before red reuses it
  if (grp > 0)
#pragma unroll
    for (int p = 0; p < 3; ++p)
#pragma unroll
      for (int q = 0; q < 3; ++q) red[grp - 1][p * 3 + q][l] = acc[p][q];
  __syncthreads();
  if (grp > 0) return;
  double* out = a.part_tr + ((size_t)b * a.nchunk + ch) * C * C;
#pragma unroll
  for (int p = 0; p < 3; ++p)
#pragma unroll
    for (int q = 0; q < 3; ++q) {
      double v = acc[p][q];
#pragma unroll
      for (int g = 0; g < NG - 1; ++g) v += red[g][p * 3 + q][l];
      const int cs = ty * 3 + p, cd = tx * 3 + q;
      if (cs < C && cd < C) out[(size_t)cs * C + cd] = v;
    }
}

// ---- transition partials: part_tr[b][chunk][c'][c] = sum_t xa f * ya --------
// CTA = (pair block, chunk, sequence); 16x16 threads, each a RT x RT tile of
// a (16 RT) x (16 RT) pair block; positions staged TS at a time.
template <int RT>
__global__ void __launch_bounds__(kMT) lmarg_tr_kernel(const LMargArgs a) {
  constexpr int PB = 16 * RT;
  constexpr int TS = 32;
  __shared__ __align__(16) double xs[TS][PB];
  __shared__ __align__(16) double ys[TS][PB];
  __shared__ double fs[TS];
  const int C = a.C, T = a.T;
  const int npb = (C + PB - 1) / PB;
  const int pr = blockIdx.x / npb, pc = blockIdx.x % npb;
  const int ch = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int Lb = seq_len(a.lengths, b, T);
  // targets t in [0, Lb-1]; chunk ch of nchunk
  const int per = (T + a.nchunk - 1) / a.nchunk;
  const int t_lo = ch * per;
  const int t_hi = min(t_lo + per, Lb);
  double acc[RT][RT];
#pragma unroll
  for (int i = 0; i < RT; ++i)
#pragma unroll
    for (int j = 0; j < RT; ++j) acc[i][j] = 0.0;
  const double lz = a.logz[b];
  const size_t rowb = (size_t)b * (T + 1);
  for (int t0 = t_lo; t0 < t_hi; t0 += TS) {
    const int n = min(TS, t_hi - t0);
    __syncthreads();
    if (tid < TS) fs[tid] = tid < n ? exp(a.xn[rowb + t0 + tid] + a.yn[rowb + t0 + tid] - lz) : 0.0;
    __syncthreads();
    for (int e = tid; e < TS * PB; e += kMT) {
      const int i = e / PB, q = e % PB;
      const int cs = pr * PB + q, cd = pc * PB + q;
      double x = 0.0, y = 0.0;
      if (i < n) {
        const size_t row = (rowb + t0 + i) * C;
        if (cs < C) x = a.xa[row + cs] * fs[i];
        if (cd < C) y = a.ya[row + cd];
      }
      xs[i][q] = x;
      ys[i][q] = y;
    }
    __syncthreads();
    for (int i = 0; i < n; ++i) {
      double xv[RT], yv[RT];
#pragma unroll
      for (int q = 0; q < RT; ++q) {
        xv[q] = xs[i][ty * RT + q];
        yv[q] = ys[i][tx * RT + q];
      }
#pragma unroll
      for (int p = 0; p < RT; ++p)
#pragma unroll
        for (int q = 0; q < RT; ++q) acc[p][q] = fma(xv[p], yv[q], acc[p][q]);
    }
  }
  double* out = a.part_tr + ((size_t)b * a.nchunk + ch) * C * C;
#pragma unroll
  for (int p = 0; p < RT; ++p)
#pragma unroll
    for (int q = 0; q < RT; ++q) {
      const int cs = pr * PB + ty * RT + p, cd = pc * PB + tx * RT + q;
      if (cs < C && cd < C) out[(size_t)cs * C + cd] = acc[p][q];
    }
}

// ---- transition partials on the float64 tensor cores (C > 64) -------------
// The same sums as lmarg_tr_kernel, as a GEMM over positions: per (pair block,
// chunk, sequence) D[c'][c] += sum_t (xa[t][c'] f_t) ya[t][c] with mma.sync
// m8n8k4 f64 (8 x 8 tiles, 4 positions per step, float64 products and sums).
// A CTA holds a 128 x 128 pair block: 8 warps of 32 x 64 (4 x 8 MMA tiles,
// 64 accumulators per lane).  Positions arrive kTMS at a time through a
// kTMN-stage cp.async pipeline (raw table rows, zero-filled past the chunk or
// the label range); f_t scales the A fragments in registers.  Rows are
// kTMR = 132 doubles apart, so that a fragment load (lane = 4 * column + step
// row) touches 16 distinct bank pairs per half warp.
constexpr int kTM = 128, kTMS = 16, kTMR = kTM + 4, kTMN = 3;

__device__ __forceinline__ void dmma_884(double& d0, double& d1, double a, double b) {
  asm volatile("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0, %1}, {%2}, {%3}, {%0, %1};"
               : "+d"(d0), "+d"(d1)
               : "d"(a), "d"(b));
}
__device__ __forceinline__ void tm_cp8(double* dst, const double* src, bool valid) {
  const unsigned d = (unsigned)__cvta_generic_to_shared(dst);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;\n" ::"r"(d), "l"(src),
               "r"(valid ? 8 : 0)
               : "memory");
}

__global__ void __launch_bounds__(kMT) lmarg_trmma_kernel(const LMargArgs a) {
  extern __shared__ __align__(16) double tsm[];
  // stage s: xs [kTMS][kTMR], ys [kTMS][kTMR], fs [kTMS]
  constexpr int kStage = 2 * kTMS * kTMR + kTMS;
  const int C = a.C, T = a.T;
  const int npb = (C + kTM - 1) / kTM;
  const int pr = blockIdx.x / npb, pc = blockIdx.x % npb;
  const int ch = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int wm = warp >> 1, wn = warp & 1;  // 4 x 2 warps of 32 x 64
  const int fr = lane & 3, fc = lane >> 2;  // fragment step row, column
  const int Lb = seq_len(a.lengths, b, T);
  const int per = (T + a.nchunk - 1) / a.nchunk;
  const int t_lo = ch * per;
  const int t_hi = min(t_lo + per, Lb);
  const int nst = t_hi > t_lo ? (t_hi - t_lo + kTMS - 1) / kTMS : 0;
  const double lz = a.logz[b];
  const size_t rowb = (size_t)b * (T + 1);
  const double* xa_b = a.xa + rowb * C;
  const double* ya_b = a.ya + rowb * C;
  // issue stage st into buffer st % kTMN (one commit group per stage, empty
  // groups past the end keep the group count uniform)
  auto issue = [&](int st) {
    if (st < nst) {
      double* xs = tsm + (st % kTMN) * kStage;
      double* ys = xs + kTMS * kTMR;
      double* fs = ys + kTMS * kTMR;
      const int t0 = t_lo + st * kTMS;
      for (int e = tid; e < kTMS * kTM; e += kMT) {
        const int i = e / kTM, q = e % kTM;
        const int cs = pr * kTM + q, cd = pc * kTM + q;
        const bool in = t0 + i < t_hi;
        const size_t row = (size_t)(t0 + i) * C;
        tm_cp8(xs + i * kTMR + q, xa_b + (in && cs < C ? row + cs : 0), in && cs < C);
        tm_cp8(ys + i * kTMR + q, ya_b + (in && cd < C ? row + cd : 0), in && cd < C);
      }
      if (tid < kTMS) {
        const int t = t0 + tid;
        fs[tid] = t < t_hi ? exp(a.xn[rowb + t] + a.yn[rowb + t] - lz) : 0.0;
      }
    }
    asm volatile("cp.async.commit_group;\n" ::: "memory");
  };
  double d[4][8][2];
#pragma unroll
  for (int mi = 0; mi < 4; ++mi)
#pragma unroll
    for (int ni = 0; ni < 8; ++ni) d[mi][ni][0] = d[mi][ni][1] = 0.0;
#pragma unroll
  for (int st = 0; st < kTMN - 1; ++st) issue(st);
  for (int st = 0; st < nst; ++st) {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(kTMN - 2) : "memory");
    __syncthreads();  // stage st is in place; the buffer of st - 1 is free
    issue(st + kTMN - 1);
    const double* xs = tsm + (st % kTMN) * kStage;
    const double* ys = xs + kTMS * kTMR;
    const double* fs = ys + kTMS * kTMR;
#pragma unroll
    for (int kk = 0; kk < kTMS / 4; ++kk) {
      const int r = (kk * 4 + fr) * kTMR;
      const double f = fs[kk * 4 + fr];
      double av[4], bv[8];
#pragma unroll
      for (int mi = 0; mi < 4; ++mi) av[mi] = xs[r + wm * 32 + mi * 8 + fc] * f;
#pragma unroll
      for (int ni = 0; ni < 8; ++ni) bv[ni] = ys[r + wn * 64 + ni * 8 + fc];
#pragma unroll
      for (int mi = 0; mi < 4; ++mi)
#pragma unroll
        for (int ni = 0; ni < 8; ++ni) dmma_884(d[mi][ni][0], d[mi][ni][1], av[mi], bv[ni]);
    }
  }
  asm volatile("cp.async.wait_group 0;\n" ::: "memory");
  // D fragment: row fc, columns 2 fr and 2 fr + 1 of each 8 x 8 tile
  double* out = a.part_tr + ((size_t)b * a.nchunk + ch) * C * C;
#pragma unroll
  for (int mi = 0; mi < 4; ++mi)
#pragma unroll
    for (int ni = 0; ni < 8; ++ni) {
      const int cs = pr * kTM + wm * 32 + mi * 8 + fc;
      const int cd = pc * kTM + wn * 64 + ni * 8 + 2 * fr;
      if (cs < C && cd < C) out[(size_t)cs * C + cd] = d[mi][ni][0];
      if (cs < C && cd + 1 < C) out[(size_t)cs * C + cd + 1] = d[mi][ni][1];
    }
}

// The transition-partial kernel for C > 64: the tensor-core GEMM unless the
// environment variable SEMICRF_TRANSITION_GEMM=fma selects the CUDA-core
// kernel (the measured comparison of the two is this switch's purpose).
bool tr_use_mma(int C) {
  if (C <= 64) return false;
  static int choice = -1;
  if (choice < 0) {
    const char* v = getenv("SEMICRF_TRANSITION_GEMM");
    choice = (v && strcmp(v, "fma") == 0) ? 0 : 1;
  }
  return choice == 1;
}

// ---- duration partials: part_db[b][split][k-1][c] = sum_t X[t,c] Y[t+k,c] ----
// CTA = (label group, split, sequence); a split is a run of whole target
// blocks.  For the target block tau (targets t0 = kTT*tau ..) and label c:
//     X[i] = Xlin[t0+i],   Y[j] = Ylin[s] * exp(mbY[blk(s)] + maX[tau] - logZ)
// for sources s = t0+1+j, so X[i] Y[i+k-1] = P(t0+i -> t0+i+k) / exp(db);
// X <= 1 and Y is bounded by a segment marginal, so both stay in range, and a
// source that underflows in Ylin is negligible beside its block's maximum.
// An item is a (label, kLG consecutive k) pair: MI items per thread.  A thread
// forms 16 targets x kLG lags per step from 16 + (16 + kLG - 1) staged values,
// so each shared-memory load serves more than five FMAs.
// The sources stay in a ring of NR = 2^m >= ny rows across the target blocks
// of a split (Ylin as stored, zero past the sequence end): each block adds
// only its 64 new rows, loaded into registers while the previous block
// computes, and the block factor G of a source is applied as the window of 31
// rows is read.  Rows 0..kDbMirror-1 are kept twice, the copy after row NR-1,
// so that a window is kDbMirror consecutive rows wherever it starts (one
// address per window, fixed offsets after it).  A window starts on a multiple
// of 16, so it reaches a second source block only when it starts at 48 mod 64,
// and then from its 16th row on.
constexpr int kLG = 16;
constexpr int kDbMirror = 32;  // >= the window's kLG + 15 rows
constexpr int kDbPF = 4;  // prefetched X and Y values per thread: kTT * cg <= kDbPF * kMT
static_assert(kTT % 16 == 0, "lmarg_db_kernel steps over targets in groups of 16");
static_assert(kTT == 64, "the ring's block arithmetic assumes 64-position blocks");

// ring rows: a power of two with room for a block's ny rows plus the next
// block's 64 new ones, which are stored while the block computes
__host__ __device__ inline int db_ring_rows(int kcap) {
  const int ny = kTT + kcap + 16;
  int r = 64;
  while (r < ny + kTT) r <<= 1;
  return r;
}

template <int MI>
__global__ void __launch_bounds__(kMT, MI == 1 ? 2 : 1) lmarg_db_kernel(const LMargArgs a) {
  extern __shared__ __align__(16) unsigned char smraw[];
  const int C = a.C, T = a.T, kcap = a.kcap, CG = a.cg;
  const int g0 = blockIdx.x * CG;
  const int cgn = min(CG, C - g0);
  const int sp = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x;
  const int nblk = (T + 1 + kTT - 1) / kTT;
  // Y rows read by a tile: targets i0 <= kTT - 16 in groups of 16, lag groups
  // k_lo <= 16*(nkg-1) + 1, window m < kLG + 15, so the last row read is
  // kTT - 16 + 16*nkg + 14 <= kTT + kcap + 13 < ny
  const int ny = kTT + kcap + 16;
  const int NR = db_ring_rows(kcap), RM = NR - 1;
  const int nq = ny / kTT + 2;  // source blocks a tile touches
  // X and G are double-buffered (block tau uses buffer (tau - tau_lo) & 1):
  // the next block is staged while this one computes, one barrier per block
  double* X = reinterpret_cast<double*>(smraw);   // [2][kTT][CG]
  double* Y = X + (size_t)2 * kTT * CG;           // [NR + kDbMirror][CG] ring, row s at s & RM
  double* G = Y + (size_t)(NR + kDbMirror) * CG;  // [2][nq][CG]
  const int nkg = (kcap + kLG - 1) / kLG;
  const int nitems = cgn * nkg;
  const int Lb = seq_len(a.lengths, b, T);
  const int ntile = (Lb + kTT - 1) / kTT;  // target blocks (targets t < Lb)
  const int per = (ntile + a.nsplit - 1) / a.nsplit;
  const int tau_lo = sp * per, tau_hi = min(tau_lo + per, ntile);
  const double lz = a.logz[b];
  const size_t rowb = (size_t)b * (T + 1);
  const double* mx_b = a.maX + (size_t)b * nblk * C + g0;
  const double* my_b = a.mbY + (size_t)b * nblk * C + g0;
  double acc[MI][kLG];
#pragma unroll
  for (int j = 0; j < MI; ++j)
#pragma unroll
    for (int q = 0; q < kLG; ++q) acc[j][q] = 0.0;
  if (tau_lo >= tau_hi) {
    // nothing of this sequence in this split: zero partials
  } else {
    // a source row of the ring (0 past the sequence end)
    auto ysrc = [&](int s, int cc) -> double {
      return (s <= Lb) ? a.lb[(rowb + s) * C + g0 + cc] : 0.0;
    };
    // the first block's sources: rows t0+1 .. t0+ny-64 now (the block's own
    // 64 new rows, t0+ny-63 .. t0+ny, arrive with the prefetch below)
    {
      const int t0 = tau_lo * kTT;
      for (int e = tid; e < (ny - kTT) * cgn; e += kMT) {
        const int j = e / cgn, cc = e % cgn;
        const int s = t0 + 1 + j, r = s & RM;
        const double v = ysrc(s, cc);
        Y[r * CG + cc] = v;
        if (r < kDbMirror) Y[(r + NR) * CG + cc] = v;
      }
    }
    // per thread: up to four X rows and four new Y rows of the next block
    constexpr int kPF = kDbPF;
    double px[kPF], py[kPF];
    auto prefetch = [&](int tau) {
      const int t0 = tau * kTT, n = min(kTT, Lb - t0);
#pragma unroll
      for (int r = 0; r < kPF; ++r) {
        const int e = tid + r * kMT;
        px[r] = py[r] = 0.0;
        if (e < kTT * cgn) {
          const int i = e / cgn, cc = e % cgn;
          if (i < n) px[r] = a.la[(rowb + t0 + i) * C + g0 + cc];
          py[r] = ysrc(t0 + ny - kTT + 1 + i, cc);
        }
      }
    };
    // block tau's X rows, its 64 new Y rows and its G factors into buffer buf
    auto stage = [&](int tau, int buf) {
      const int t0 = tau * kTT;
      double* Xb = X + (size_t)buf * kTT * CG;
      double* Gb = G + (size_t)buf * nq * CG;
#pragma unroll
      for (int r = 0; r < kPF; ++r) {
        const int e = tid + r * kMT;
        if (e < kTT * cgn) {
          const int i = e / cgn, cc = e % cgn;
          Xb[i * CG + cc] = px[r];
          const int row = (t0 + ny - kTT + 1 + i) & RM;
          Y[row * CG + cc] = py[r];
          if (row < kDbMirror) Y[(row + NR) * CG + cc] = py[r];
        }
      }
      for (int e = tid; e < nq * cgn; e += kMT) {
        const int q = e / cgn, cc = e % cgn;
        const int beta = tau + q;
        double gv = 0.0;
        if (beta < nblk) {
          const double rx = mx_b[(size_t)tau * C + cc], ry = my_b[(size_t)beta * C + cc];
          if (rx > -INFINITY && ry > -INFINITY) {
            const double ex = ry + rx - lz;
            // beyond this the factored tile loses terms (or clamps): the sequence
            // is recomputed term by term by lmarg_db_fix_kernel
            if (ex > kDbFlag) a.dbflag[b] = 1;
            gv = exp(fmin(ex, 700.0));
          }
        }
        Gb[q * CG + cc] = gv;
      }
    };
    prefetch(tau_lo);
    stage(tau_lo, 0);
    if (tau_lo + 1 < tau_hi) prefetch(tau_lo + 1);
    for (int tau = tau_lo; tau < tau_hi; ++tau) {
      const int t0 = tau * kTT;
      const int n = min(kTT, Lb - t0);
      const int cur = (tau - tau_lo) & 1;
      // block tau is staged, and every read of block tau - 1 (the other
      // buffer) is done; block tau + 1's new Y rows lie outside block tau's
      // ny rows of the ring (NR >= ny + kTT)
      __syncthreads();
      if (tau + 1 < tau_hi) {
        stage(tau + 1, cur ^ 1);
        if (tau + 2 < tau_hi) prefetch(tau + 2);  // in flight while this block computes
      }
      const double* Xc = X + (size_t)cur * kTT * CG;
      const double* Gc = G + (size_t)cur * nq * CG;
#pragma unroll
      for (int jt = 0; jt < MI; ++jt) {
        const int it = tid + jt * kMT;
        if (it < nitems) {
          const int cc = it % cgn, kg = it / cgn;
          const int k_lo = 1 + kLG * kg;
          // target i pairs with Y[i + k - 1]: for targets i0 .. i0+15 the
          // window y[m] = Y[i0 + k_lo - 1 + m], m < kLG + 15, covers all kLG
          // lags (X is zero beyond the last target, and lags past kcap are
          // discarded below)
          for (int i0 = 0; i0 < n; i0 += 16) {
            const int j0 = i0 + k_lo - 1;  // a multiple of 16
            // source block of row j: (1 + j) >> 6; the window's first block,
            // and the factor of its rows 15.. (the next block's when j0 = 48 mod 64)
            const int q0 = (1 + j0) >> 6;
            const double gl = Gc[q0 * CG + cc];
            const double gh = (j0 & 63) == 48 ? Gc[(q0 + 1) * CG + cc] : gl;
            const double* yw = Y + ((t0 + 1 + j0) & RM) * CG + cc;
            double y[kLG + 15];
#pragma unroll
            for (int m = 0; m < kLG + 15; ++m) y[m] = yw[m * CG] * (m < 15 ? gl : gh);
            const double* xw = Xc + i0 * CG + cc;
#pragma unroll
            for (int d = 0; d < 16; ++d) {
              const double xd = xw[d * CG];
#pragma unroll
              for (int q = 0; q < kLG; ++q) acc[jt][q] = fma(xd, y[d + q], acc[jt][q]);
            }
          }
        }
      }
    }
  }
  double* out = a.part_db + ((size_t)b * a.nsplit + sp) * (size_t)kcap * C;
#pragma unroll
  for (int jt = 0; jt < MI; ++jt) {
    const int it = tid + jt * kMT;
    if (it < nitems) {
      const int cc = it % cgn, kg = it / cgn;
#pragma unroll
      for (int q = 0; q < kLG; ++q) {
        const int k = 1 + kLG * kg + q;
        if (k <= kcap) out[(size_t)(k - 1) * C + g0 + cc] = acc[jt][q];
      }
    }
  }
}

// ---- duration partials of flagged sequences, term by term ---------------------
// When the scores inside a 64-position block span more than the float64
// exponent range (very large emission scores), the block-factored tiles above
// lose or clamp terms; lmarg_db_kernel flags such a sequence.  Its partials are
// recomputed here from the saved chain tables in the log domain,
//   part_db[b][0][k-1][c] = sum_t exp(la[t,c] + lb[t+k,c] - logZ),
//   la = log xA + xn + ps - cum (t < len),  lb = log yA + yn + cum + pe (t+k <= len),
// and the other splits are zeroed.  Unflagged sequences return at once.
__global__ void __launch_bounds__(kMT) lmarg_db_fix_kernel(const LMargArgs a) {
  const int b = blockIdx.y;
  if (a.dbflag[b] == 0) return;
  const int C = a.C, T = a.T, kcap = a.kcap;
  const int it = blockIdx.x * kMT + threadIdx.x;
  if (it >= kcap * C) return;
  const int k = 1 + it / C, c = it % C;
  const int Lb = seq_len(a.lengths, b, T);
  const double lz = a.logz[b];
  const size_t row0 = (size_t)b * (T + 1);
  const float* cum_b = a.cum + row0 * C;
  double sum = 0.0;
  for (int t = 0; t < Lb && t + k <= Lb; ++t) {
    const int s = t + k;
    const double x = a.xA[(row0 + t) * C + c], y = a.yA[(row0 + s) * C + c];
    if (!(x > 0.0) || !(y > 0.0)) continue;
    const double ps = a.ps ? (double)a.ps[((size_t)b * T + t) * C + c] : 0.0;
    const double pe = a.pe ? (double)a.pe[((size_t)b * T + s - 1) * C + c] : 0.0;
    const double la = log(x) + a.xn[row0 + t] + ps - (double)cum_b[(size_t)t * C + c];
    const double lb = log(y) + a.yn[row0 + s] + (double)cum_b[(size_t)s * C + c] + pe;
    sum += exp(la + lb - lz);
  }
  double* out = a.part_db + (size_t)b * a.nsplit * kcap * C;
  out[(size_t)(k - 1) * C + c] = sum;
  for (int sp = 1; sp < a.nsplit; ++sp) out[((size_t)sp * kcap + k - 1) * C + c] = 0.0;
}

// ---- fixed-order reduction over sequences and chunks -------------------------
// One warp per output: lane l sums the terms (b, chunk) = l, l+32, ... in
// order, then a fixed shuffle tree adds the lanes.
__global__ void __launch_bounds__(kMT) lmarg_reduce_kernel(const LMargArgs a, float* grad_tr,
                                                            float* grad_db) {
  const int C = a.C, K = a.K, kcap = a.kcap;
  const int ntr = C * C, ndb = K * C;
  const int lane = threadIdx.x & 31;
  const int warp = (blockIdx.x * kMT + threadIdx.x) >> 5;
  const int nwarps = (gridDim.x * kMT) >> 5;
  for (int o = warp; o < ntr + ndb; o += nwarps) {
    double s = 0.0;
    if (o < ntr) {
      const int nterm = a.B * a.nchunk;
      for (int q = lane; q < nterm; q += 32) {
        const int b = q / a.nchunk;
        s = fma((double)a.grad_output[b], a.part_tr[(size_t)q * ntr + o], s);
      }
    } else {
      const int j = (o - ntr) / C, c = (o - ntr) % C;
      // duration index j collects k with min(k, K-1) == j
      const int k = (K == 1) ? 1 : j;
      if (k >= 1 && k <= kcap) {
        const int nterm = a.B * a.nsplit;
        for (int q = lane; q < nterm; q += 32) {
          const int b = q / a.nsplit;
          s = fma((double)a.grad_output[b],
                  a.part_db[(size_t)q * kcap * C + (size_t)(k - 1) * C + c], s);
        }
      }
    }
#pragma unroll
    for (int w = 16; w > 0; w >>= 1) s += __shfl_xor_sync(0xffffffffu, s, w);
    if (lane == 0) {
      if (o < ntr) {
        grad_tr[o] = (float)(exp((double)a.tr[o]) * s);
      } else {
        const int j = (o - ntr) / C, c = (o - ntr) % C;
        grad_db[o - ntr] = (float)(s * exp((double)a.db[(size_t)j * C + c]));
      }
    }
  }
}


}  // namespace

LMargPlan lmarg_plan(int B, int T, int K, int C) {
  LMargPlan p{};
  const int kcap = K > 1 ? K - 1 : 1;
  const int sms = device_sm_count();
  // transition partials
  const int pb = C <= 32 ? 32 : (tr_use_mma(C) ? kTM : 64);
  const int npb = (C + pb - 1) / pb;
  // two CTAs per SM for the CUDA-core kernels; one wave of one CTA per SM
  // for the tensor-core kernel (its 64 accumulators per lane fill the registers)
  int nch = pb == kTM ? sms / (B * npb * npb)
                      : (2 * sms + B * npb * npb - 1) / (B * npb * npb);
  const int maxch = (T + 255) / 256;
  if (nch > maxch) nch = maxch;
  if (nch < 1) nch = 1;
  p.nchunk = nch;
  // duration partials: label group sized so that the staging fits two CTAs
  // per SM with one item per thread where possible, else one CTA with two
  const int ny = kTT + kcap + 16;
  const int nq = ny / kTT + 2;
  const size_t per_label = 8 * (size_t)(2 * kTT + db_ring_rows(kcap) + kDbMirror + 2 * nq);
  const int nkg = (kcap + kLG - 1) / kLG;
  auto fit = [&](size_t smem, int items) {
    long cg = (long)(smem / per_label);
    const long ci = (long)items * kMT / nkg;
    if (cg > ci) cg = ci;
    if (cg > C) cg = C;
    if (cg > kDbPF * kMT / kTT) cg = kDbPF * kMT / kTT;  // one block's rows prefetched
    return (int)cg;
  };
  int cg = fit(110 * 1024, 1);
  p.mi = 1;
  if (cg < 1 || (cg < C && fit(200 * 1024, 2) >= 2 * cg)) {
    cg = fit(200 * 1024, 2);
    p.mi = 2;
  }
  if (cg < 1) cg = 1;
  p.cg = cg;
  p.ncg = (C + cg - 1) / cg;
  // about six waves of resident CTAs, so that the sequences' unequal lengths
  // even out (measured at configuration 2: 1.13 ms backward with two waves,
  // 1.06 ms with six), but at least four target blocks per CTA (the ring fill
  // is a fixed cost per CTA)
  const int target = (p.mi == 1 ? 12 : 6) * sms;
  int nsp = (target + B * p.ncg - 1) / (B * p.ncg);
  const int maxsp = (T + kTT - 1) / kTT;
  const int capsp = maxsp / 4 > 1 ? maxsp / 4 : 1;
  if (nsp > capsp) nsp = capsp;
  if (nsp < 1) nsp = 1;
  p.nsplit = nsp;
  p.nblk = (T + 1 + kTT - 1) / kTT;
  p.db_smem = per_label * cg;
  p.ok = (size_t)cg * nkg <= (size_t)p.mi * kMT && p.db_smem <= 227 * 1024;
  return p;
}

cudaError_t launch_lmarg(const LMargArgs& a, float* grad_tr, float* grad_db, cudaStream_t s) {
  if (a.B <= 0) return cudaSuccess;
  const LMargPlan p = lmarg_plan(a.B, a.T, a.K, a.C);
  if (!p.ok || p.nchunk != a.nchunk || p.nsplit != a.nsplit || p.cg != a.cg)
    return cudaErrorInvalidValue;
  const int gmax = device_sm_count() * 16;
  const dim3 gpb(p.nblk, (a.C + kPG - 1) / kPG, a.B);
  cudaError_t e;
  if (posblk_pairs(a)) {
    e = cudaFuncSetAttribute(lmarg_posblk_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             posblk_smem(a.C));
    if (e != cudaSuccess) return e;
    lmarg_posblk_kernel<2><<<gpb, kMT, posblk_smem(a.C), s>>>(a);
  } else {
    e = cudaFuncSetAttribute(lmarg_posblk_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             posblk_smem(a.C));
    if (e != cudaSuccess) return e;
    lmarg_posblk_kernel<1><<<gpb, kMT, posblk_smem(a.C), s>>>(a);
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  int g;
  if (a.C <= 24) {
    lmarg_tr24_kernel<<<dim3(1, a.nchunk, a.B), kMT, 0, s>>>(a);
  } else if (a.C <= 32) {
    const int npb = (a.C + 31) / 32;
    lmarg_tr_kernel<2><<<dim3(npb * npb, a.nchunk, a.B), kMT, 0, s>>>(a);
  } else if (tr_use_mma(a.C)) {
    const int npb = (a.C + kTM - 1) / kTM;
    const int smem = kTMN * (2 * kTMS * kTMR + kTMS) * 8;
    e = cudaFuncSetAttribute(lmarg_trmma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             smem);
    if (e != cudaSuccess) return e;
    lmarg_trmma_kernel<<<dim3(npb * npb, a.nchunk, a.B), kMT, smem, s>>>(a);
  } else {
    const int npb = (a.C + 63) / 64;
    lmarg_tr_kernel<4><<<dim3(npb * npb, a.nchunk, a.B), kMT, 0, s>>>(a);
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const dim3 gdb(p.ncg, a.nsplit, a.B);
  if (p.mi == 1) {
    e = cudaFuncSetAttribute(lmarg_db_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)p.db_smem);
    if (e != cudaSuccess) return e;
    lmarg_db_kernel<1><<<gdb, kMT, p.db_smem, s>>>(a);
  } else {
    e = cudaFuncSetAttribute(lmarg_db_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)p.db_smem);
    if (e != cudaSuccess) return e;
    lmarg_db_kernel<2><<<gdb, kMT, p.db_smem, s>>>(a);
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  lmarg_db_fix_kernel<<<dim3((a.kcap * a.C + kMT - 1) / kMT, a.B), kMT, 0, s>>>(a);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const int nout = a.C * a.C + a.K * a.C;
  g = (nout * 32 + kMT - 1) / kMT;
  if (g > gmax) g = gmax;
  lmarg_reduce_kernel<<<g, kMT, 0, s>>>(a, grad_tr, grad_db);
  return cudaGetLastError();
}

}  // namespace semicrf
