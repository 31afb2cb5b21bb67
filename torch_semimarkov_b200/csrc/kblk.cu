// kblk.cu -- (K, C, C) transitions, log semiring: the blocked chain.
//
// The recurrences are those of kcc.cu (pytorch_reference.py:87-111 with
// transition[k] per duration, :213 and :437-446):
//   alpha[t,c] = ct[t,c] + (+)_{k,c'} ( alpha[t-k,c'] + tr[k][c',c] + db[k,c] + dt[t-k,c] )
//   beta[s,c'] = (+)_{k,c} ( tr[k][c',c] + db[k,c] + dt[s,c] + ct[s+k,c] + beta[s+k,c] )
// with ct[t,c] = cum[t,c] + pe[t-1,c], dt[s,c] = ps[s,c] - cum[s,c], alpha[0] = 0,
// beta[len] = 0, durations k = 1 .. K-1.  Both directions are written in the
// chain's own position index rho (rho = t forward, rho = len - s backward), in
// which the source of duration k is rho - k.
//
// Positions are processed in blocks of P.  With the per-label constant
// fk[c] = max_{k,c'} (tr[k][c',c] + db[k,c]) the weights
//   xf[k][m][l] = exp(tr[k][m][l] + db[k][l] - fk[l])   (forward, m = source label)
//   xb[k][m][l] = exp(tr[k][l][m] + db[k][m] - fk[m])   (backward, m = next label)
// are at most 1, and every source enters in float64 linear form relative to a
// per-label frame fixed at the start of its block:
//   forward   a[s,m] = exp(alpha[s,m] - n_s),  y[s,l] = exp(n_s + dt[s,l] + fk[l] - F[l])
//             exp(alpha[t,l] - ct[t,l] - F[l]) = sum_{s,m} xf[t-s][m][l] a[s,m] y[s,l] w[l]
//   backward  g[u,m] = exp(beta[u,m] + ct[u,m] + fk[m] - H[m]),  v[s,m] = exp(dt[s,m] + H[m] - Rb)
//             exp(beta[s,l] - Rb) = sum_m v[s,m] sum_u xb[u-s][m][l] g[u,m] w[m]
// where n_s is the row maximum of alpha, F (H) the frame of the target block
// and w = exp(frame of the source's block - frame of the target block).  A
// frame is taken from the last row of the previous block, so within a block
// the factors only drift by the emissions of P positions; values that fall
// below the float64 range are dropped (their weight relative to the row's
// maximum is below e^-700).
//
// Per block, with all threads of the CTA:
//  1. far sums: every source in an earlier block.  The work of output label l
//     is (contracted label m) x (source block q) units; one unit is the P x P
//     Toeplitz tile out[j] += sum_r x[D + j - r][m][l] z[r] (D = block
//     distance), evaluated from a register window of 2P-1 weights that slides
//     by P between consecutive source blocks, so each weight is loaded once
//     per block and used P times.  Units are split evenly over the threads of
//     each label; a fixed-order sum over the threads gives the block's
//     pending values.
//  2. the P rows in order: a row's source factors are its pending values
//     times a per-block factor, and its contributions to the later rows of
//     the block (durations 1 .. P-1) are one C-term dot product per (target,
//     label) with weights held in registers; one barrier per row.
//  3. the block's log tables and row maxima, in parallel.
// The tables written are those of kcc_chain_kernel: log alpha and its row
// maxima (forward), log beta (backward), log Z and the ring checkpoints.

#include <cooperative_groups.h>

#include "semicrf_internal.cuh"

namespace semicrf {

namespace cg = cooperative_groups;

namespace {

constexpr int kBT = 256;  // threads per CTA
constexpr int kBP = 16;   // positions per block
constexpr size_t kBSmemMax = 220 * 1024;

__device__ __forceinline__ int bseq_len(const int64_t* lengths, int b, int T) {
  const long long l = lengths[b];
  return l < 0 ? 0 : (l > T ? T : (int)l);
}

__device__ __forceinline__ int floor_div(int a, int b) {
  return a >= 0 ? a / b : -((-a + b - 1) / b);
}

// Shared memory of the blocked chain (offsets in doubles, each even).
struct BlkPlan {
  int nbr, R;
  size_t ra, ry, fn, fd, wq, pend, part, ctb, dtb, kap, vb, lv, fk, vals, red, total;
};
__host__ __device__ inline BlkPlan blk_plan(int C, int K, int P) {
  BlkPlan p{};
  p.nbr = (K - 1 + P - 1) / P + 2;  // far source blocks + the current one + 1
  p.R = p.nbr * P;
  size_t o = 0;
  auto take = [&](size_t n) {
    const size_t r = o;
    o += (n + 1) & ~size_t(1);
    return r;
  };
  p.ra = take((size_t)p.R * C);    // forward a rows / backward g rows
  p.ry = take((size_t)p.R * C);    // forward y rows
  p.fn = take(p.nbr);              // frame of each block in the ring: scalar part N
  p.fd = take((size_t)p.nbr * C);  // and per-label part (dt or ct of its reference row)
  p.wq = take((size_t)p.nbr * C);  // rebase factor per far source block
  p.pend = take((size_t)P * C);    // pending values of the block's positions
  p.part = take((size_t)P * kBT);  // per-thread far sums
  p.ctb = take((size_t)P * C);
  p.dtb = take((size_t)P * C);
  p.kap = take((size_t)P * C);     // factor from pending value to source factor
  p.vb = take((size_t)P * C);      // forward y / backward target factors v
  p.lv = take((size_t)P * C);      // the block's log values
  p.fk = take(C);
  p.vals = take(C);
  p.red = take(64);
  p.total = o;
  return p;
}

constexpr int kRegC = 32;  // largest C whose near weights are kept in registers
constexpr int kBMaxQ = 8;  // largest cluster per chain (the portable cluster size)

// Frames.  Block tau has a scalar N and per-label offsets fd[l], taken from
// the row before the block (its reference row; position 0 or len for the
// first block): forward N = max_l alpha, fd = dt of that row, and
//   F[l] = N + fd[l] + fk[l]    a[s,m] = pend[s,m] exp(ct[s,m] + fd[m] + fk[m])
//                               y[s,l] = exp(dt[s,l] - fd[l])
// backward N = max_l beta, fd = ct of that row, rb = max_m (dt[first,m] + fd[m] + fk[m]),
//   H[m] = N + fd[m] + fk[m]    g[u,m] = pend[u,m] exp(rb + ct[u,m] - fd[m])
//                               v[s,m] = exp(dt[s,m] + fd[m] + fk[m] - rb)
// where pend is the row's sum relative to its frame, so alpha = N + log a and
// beta = N + fd - ct + log g.  The kernel accumulates the factors a (g)
// directly: every contribution to a row is multiplied by the row's
// exp(ct + fd + fk) (exp(rb + ct - fd)), so no log or exp lies between the
// rows of a block.  The log tables are written per block, after its rows.
template <int P, int CR>
__global__ void __launch_bounds__(kBT, 1) kblk_chain_kernel(const KccArgs a, int Q) {
  extern __shared__ __align__(16) double bsm[];
  const int C = a.C, K = a.K, T = a.T, kcap = a.kcap;
  // Q CTAs (one cluster when Q > 1) per sequence and direction: they split the
  // far sums and repeat the rest, so every rank holds the same state; rank 0
  // writes the outputs
  const int b = blockIdx.x / Q, rank = blockIdx.x % Q, dir = blockIdx.y, tid = threadIdx.x;
  const bool out0 = rank == 0;
  const int lane = tid & 31, warp = tid >> 5;
  const int Lb = bseq_len(a.lengths, b, T);
  const BlkPlan pl = blk_plan(C, K, P);
  const int NBR = pl.nbr;
  double* ra = bsm + pl.ra;
  double* ry = bsm + pl.ry;
  double* fN = bsm + pl.fn;
  double* fd = bsm + pl.fd;
  double* wq = bsm + pl.wq;
  double* pend = bsm + pl.pend;
  double* part = bsm + pl.part;
  double* ctb = bsm + pl.ctb;
  double* dtb = bsm + pl.dtb;
  double* kap = bsm + pl.kap;
  double* vb = bsm + pl.vb;
  double* lv = bsm + pl.lv;
  double* fk = bsm + pl.fk;
  double* vals = bsm + pl.vals;
  double* red = bsm + pl.red;  // [32]: maximum of the last row of the previous block; [33]: rb
  const float* cum_b = a.cum + (size_t)b * (T + 1) * C;
  const float* ps_b = a.ps ? a.ps + (size_t)b * T * C : nullptr;
  const float* pe_b = a.pe ? a.pe + (size_t)b * T * C : nullptr;
  const double* X = dir == 0 ? a.pr.xf : a.pr.xb;
  const size_t CC = (size_t)C * C;
  // exp of a frame exponent; near the float64 range the blocked factoring is no
  // longer exact, so the flag asks for the per-position fallback chain
  auto cexp = [&](double x) -> double {
    if (x > 600.0 && a.kflag) *a.kflag = 1;
    return exp(fmin(x, 700.0));
  };

  for (int i = tid; i < C; i += kBT) fk[i] = a.pr.fk[i];
  if (dir == 0 && a.ref_ckpt && out0) {
    float* rc = a.ref_ckpt + (size_t)b * a.nref * K * C;
    for (size_t i = tid; i < (size_t)a.nref * K * C; i += kBT)
      rc[i] = (i < (size_t)C) ? 0.f : kRefNegInf;
  }
  if (tid == 0) red[32] = 0.0;
  __syncthreads();

  const int G = kBT / C, ell = tid % C, sig = tid / C;
  const bool act = sig < G;
  const int nblk = Lb / P + 1;
  const int nnear = (P - 1) * C;  // (duration 1..P-1, label) items of the in-block contributions
  for (int tau = 0; tau < nblk; ++tau) {
    const int s0 = tau * P, fs = tau % NBR;
    // this block's frame from its reference row (the previous block's last row,
    // still in ctb / dtb); a row of -inf keeps the previous frame
    {
      const double nr = red[32];
      const bool fresh = tau == 0 || nr > -INFINITY;
      for (int l = tid; l < C; l += kBT) {
        double d;
        if (tau == 0) {
          const double cu = cum_b[(size_t)(dir == 0 ? 0 : Lb) * C + l];
          d = dir == 0 ? ((ps_b && T > 0) ? (double)ps_b[l] : 0.0) - cu
                       : cu + ((pe_b && Lb >= 1) ? (double)pe_b[(size_t)(Lb - 1) * C + l] : 0.0);
        } else {
          d = fresh ? (dir == 0 ? dtb : ctb)[(P - 1) * C + l] : fd[((tau - 1) % NBR) * C + l];
        }
        fd[fs * C + l] = d;
      }
      if (tid == 0) fN[fs] = tau == 0 ? 0.0 : (fresh ? nr : fN[(tau - 1) % NBR]);
    }
    __syncthreads();
    const double N = fN[fs];
    // the block's input terms; pending values start at zero
    for (int i = tid; i < P * C; i += kBT) {
      const int j = i / C, l = i % C, rho = s0 + j;
      double cv = 0.0, dv = 0.0;
      if (rho <= Lb) {
        const int t = dir == 0 ? rho : Lb - rho;
        const double cu = cum_b[(size_t)t * C + l];
        cv = cu + ((pe_b && t >= 1) ? (double)pe_b[(size_t)(t - 1) * C + l] : 0.0);
        dv = ((ps_b && t < T) ? (double)ps_b[(size_t)t * C + l] : 0.0) - cu;
      }
      ctb[i] = cv;
      dtb[i] = dv;
      pend[i] = rho == 0 ? 1.0 : 0.0;  // position 0: alpha = 0 (beta = 0), factor 1
    }
    const int bmin = max(0, floor_div(s0 - kcap, P));
    const int nq = tau - bmin;  // far source blocks bmin .. tau-1
    for (int i = tid; i < nq * C; i += kBT) {
      const int q = (bmin + i / C) % NBR, l = i % C;
      wq[q * C + l] = cexp(fN[q] - N + fd[q * C + l] - fd[fs * C + l]);
    }
    __syncthreads();
    double rb = 0.0;
    if (dir == 1) {
      if (warp == 0) {
        const int jf = tau == 0 ? 1 : 0;
        double mx = -INFINITY;
        if (s0 + jf <= Lb)
          for (int m = lane; m < C; m += 32) mx = fmax(mx, dtb[jf * C + m] + fd[fs * C + m] + fk[m]);
        for (int o = 16; o > 0; o >>= 1) mx = fmax(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        if (lane == 0) red[33] = mx;
      }
      __syncthreads();
      rb = red[33];
    }
    // per-row factors of the block
    for (int i = tid; i < P * C; i += kBT) {
      const int j = i / C, l = i % C;
      const double dd = fd[fs * C + l];
      if (dir == 0) {
        kap[i] = cexp(ctb[i] + dd + fk[l]);
        const double y = cexp(dtb[i] - dd);
        vb[i] = y;
        ry[(size_t)(fs * P + j) * C + l] = y;
      } else {
        const bool ok = rb > -INFINITY;
        vb[i] = ok ? cexp(dtb[i] + dd + fk[l] - rb) : 0.0;
        kap[i] = ok ? cexp(rb + ctb[i] - dd) : 0.0;
      }
    }
    __syncthreads();

    // 1. far sums
    if (nq > 0) {
      double out[P];
#pragma unroll
      for (int j = 0; j < P; ++j) out[j] = 0.0;
      if (act) {
        const int U = C * nq;
        const int QG = Q * G, slot = rank * G + sig;  // this thread's share of the cluster's
        const int u0 = (int)((long long)slot * U / QG), u1 = (int)((long long)(slot + 1) * U / QG);
        double d[2 * P - 1], nx[P];
        // unit u = m * nq + (q - bmin), advanced without divisions
        int m = u0 / nq, qi = u0 % nq;
        for (int u = u0; u < u1; ++u) {
          if (u > u0 && ++qi == nq) {
            qi = 0;
            ++m;
          }
          const int q = bmin + qi, qs = q % NBR;
          const int D = (tau - q) * P;
          const double* xc = X + (size_t)m * C + ell;
          if (u > u0 && qi != 0) {  // same label as the previous unit, next source block
#pragma unroll
            for (int i = 2 * P - 2; i >= P; --i) d[i] = d[i - P];
#pragma unroll
            for (int i = 0; i < P; ++i) d[i] = nx[i];
          } else {
#pragma unroll
            for (int i = 0; i < 2 * P - 1; ++i) {
              const int k = D - P + 1 + i;
              d[i] = k <= kcap ? __ldcg(xc + (size_t)k * CC) : 0.0;
            }
          }
          // the next unit's new weights, in flight during this unit's tile
          if (u + 1 < u1 && qi + 1 < nq) {
#pragma unroll
            for (int i = 0; i < P; ++i) {
              const int k = D - 2 * P + 1 + i;
              nx[i] = (k >= 1 && k <= kcap) ? __ldcg(xc + (size_t)k * CC) : 0.0;
            }
          }
          const int base = qs * P;
          double z[P];
          if (dir == 0) {
            const double w = wq[qs * C + ell];
#pragma unroll
            for (int r = 0; r < P; ++r)
              z[r] = ra[(size_t)(base + r) * C + m] * ry[(size_t)(base + r) * C + ell] * w;
#pragma unroll
            for (int r = 0; r < P; ++r)
#pragma unroll
              for (int j = 0; j < P; ++j) out[j] = fma(d[P - 1 + j - r], z[r], out[j]);
          } else {
            const double w = wq[qs * C + m];
#pragma unroll
            for (int r = 0; r < P; ++r) z[r] = ra[(size_t)(base + r) * C + m] * w;
            double acc[P];
#pragma unroll
            for (int j = 0; j < P; ++j) acc[j] = 0.0;
#pragma unroll
            for (int r = 0; r < P; ++r)
#pragma unroll
              for (int j = 0; j < P; ++j) acc[j] = fma(d[P - 1 + j - r], z[r], acc[j]);
#pragma unroll
            for (int j = 0; j < P; ++j) out[j] = fma(vb[j * C + m], acc[j], out[j]);
          }
        }
      }
#pragma unroll
      for (int j = 0; j < P; ++j) part[j * kBT + tid] = out[j];
      __syncthreads();
      for (int i = tid; i < P * C; i += kBT) {
        const int j = i / C, l = i % C;
        double s = 0.0;
        for (int g = 0; g < G; ++g) s += part[j * kBT + g * C + l];
        if (Q == 1)
          pend[i] = s * kap[i];
        else
          lv[i] = s;  // this rank's share, summed over the ranks in rank order below
      }
      if (Q > 1) {
        cg::cluster_group cl = cg::this_cluster();
        cl.sync();
        for (int i = tid; i < P * C; i += kBT) {
          double s = 0.0;
          for (int r = 0; r < Q; ++r) s += cl.map_shared_rank(lv, r)[i];
          pend[i] = s * kap[i];
        }
        cl.sync();  // every rank has read lv before its tables overwrite it
      } else {
        __syncthreads();
      }
    }

    // 2. the block's rows in order.  pend holds a row's source factors (a or
    // g) once the row is complete.  Item i = tid + r * kBT of row j is the
    // contribution of row j to row j + k (k = 1 + i / C) at label i % C; its
    // C weights do not depend on j and stay in registers for the block (CR >
    // 0: C <= CR).  One barrier per row.
    const int last = min(P - 1, Lb - s0);
    if constexpr (CR > 0) {
      constexpr int NREP = ((P - 1) * CR + kBT - 1) / kBT;
      double w[NREP][CR];
      int kr[NREP], lr[NREP];
      bool vr[NREP];
#pragma unroll
      for (int rep = 0; rep < NREP; ++rep) {
        const int i = tid + rep * kBT;
        kr[rep] = 1 + i / C;
        lr[rep] = i % C;
        vr[rep] = i < nnear && kr[rep] <= kcap;
#pragma unroll
        for (int m = 0; m < CR; ++m)
          w[rep][m] = (vr[rep] && m < C) ? __ldg(X + ((size_t)kr[rep] * C + m) * C + lr[rep]) : 0.0;
      }
      for (int j = 0; j <= last; ++j) {
        const double* pj = pend + j * C;
#pragma unroll
        for (int rep = 0; rep < NREP; ++rep) {
          const int jj = j + kr[rep], l = lr[rep];
          if (vr[rep] && jj <= last) {
            double s4[4] = {0.0, 0.0, 0.0, 0.0};
            if (dir == 0) {
#pragma unroll
              for (int m = 0; m < CR; ++m)
                if (m < C) s4[m & 3] = fma(pj[m], w[rep][m], s4[m & 3]);
              pend[jj * C + l] +=
                  kap[jj * C + l] * vb[j * C + l] * ((s4[0] + s4[1]) + (s4[2] + s4[3]));
            } else {
              const double* vj = vb + jj * C;
#pragma unroll
              for (int m = 0; m < CR; ++m)
                if (m < C) s4[m & 3] = fma(pj[m] * vj[m], w[rep][m], s4[m & 3]);
              pend[jj * C + l] += kap[jj * C + l] * ((s4[0] + s4[1]) + (s4[2] + s4[3]));
            }
          }
        }
        __syncthreads();
      }
    } else {
      for (int j = 0; j <= last; ++j) {
        const double* pj = pend + j * C;
        for (int i = tid; i < nnear; i += kBT) {
          const int k = 1 + i / C, l = i % C, jj = j + k;
          if (k > kcap || jj > last) continue;
          const double* xk = X + (size_t)k * CC + l;
          const double* vj = vb + jj * C;
          auto am = [&](int m) { return dir == 0 ? pj[m] : pj[m] * vj[m]; };
          double s0a = 0.0, s1a = 0.0, s2a = 0.0, s3a = 0.0;
          int m = 0;
          for (; m + 3 < C; m += 4) {
            s0a = fma(am(m), __ldg(xk + (size_t)m * C), s0a);
            s1a = fma(am(m + 1), __ldg(xk + (size_t)(m + 1) * C), s1a);
            s2a = fma(am(m + 2), __ldg(xk + (size_t)(m + 2) * C), s2a);
            s3a = fma(am(m + 3), __ldg(xk + (size_t)(m + 3) * C), s3a);
          }
          for (; m < C; ++m) s0a = fma(am(m), __ldg(xk + (size_t)m * C), s0a);
          pend[jj * C + l] += kap[jj * C + l] * (dir == 0 ? vb[j * C + l] : 1.0) *
                              ((s0a + s1a) + (s2a + s3a));
        }
        __syncthreads();
      }
    }

    // 3. the block's log tables and row maxima
    const int nrow = last + 1;
    for (int i = tid; i < nrow * C; i += kBT) {
      const int j = i / C, l = i % C, rho = s0 + j;
      const int t = dir == 0 ? rho : Lb - rho;
      const double pv = pend[i];
      if (!(pv < INFINITY) && a.kflag) *a.kflag = 1;  // an overflowed row (or NaN)
      ra[(size_t)(fs * P + j) * C + l] = pv;
      double v = 0.0;
      if (rho > 0)
        v = pv > 0.0 ? (dir == 0 ? N : N + fd[fs * C + l] - ctb[i]) + log(pv) : -INFINITY;
      lv[i] = v;
      if (!out0) continue;
      if (dir == 0) {
        if (a.alpha) a.alpha[((size_t)b * (T + 1) + t) * C + l] = v;
        if (a.ref_ckpt) {
          const int S = a.sref;
          const int ic = (t + S - 1) / S;
          if (ic < a.nref && (long long)ic * S <= Lb && (long long)ic * S - t < K)
            a.ref_ckpt[(((size_t)b * a.nref + ic) * K + (t % K)) * C + l] =
                v > -INFINITY ? (float)v : kRefNegInf;
        }
      } else if (a.beta) {
        a.beta[((size_t)b * (T + 1) + t) * C + l] = v;
      }
    }
    __syncthreads();
    for (int j = warp; j < nrow; j += kBT / 32) {
      double mx = -INFINITY;
      for (int l = lane; l < C; l += 32) mx = fmax(mx, lv[j * C + l]);
      for (int o = 16; o > 0; o >>= 1) mx = fmax(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      if (lane == 0) {
        const int t = dir == 0 ? s0 + j : Lb - (s0 + j);
        if (dir == 0 && a.amax && out0) a.amax[(size_t)b * (T + 1) + t] = mx;
        if (j == P - 1) red[32] = mx;
      }
    }
    if (s0 + last == Lb)
      for (int l = tid; l < C; l += kBT) vals[l] = lv[last * C + l];
    __syncthreads();
  }
  if (dir == 0 && tid == 0 && out0) {
    double lz = (double)kRefNegInf;
    if (Lb > 0) {
      double M = -INFINITY;
      for (int q = 0; q < C; ++q) M = fmax(M, vals[q]);
      if (M > -INFINITY) {
        double Sz = 0.0;
        for (int q = 0; q < C; ++q) Sz += exp(vals[q] - M);
        lz = M + log(Sz);
      }
    }
    if (a.logz) a.logz[b] = lz;
    if (a.partition) a.partition[b] = (float)lz;
  }
}

// fk[c] = max over durations 1 .. K-1 and source labels of tr + db (the
// prepared tdf), 0 when that is -inf so the weights of the label become 0
__global__ void kblk_fk_kernel(int K, int C, KccPrep pr) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  double m = -INFINITY;
  for (int k = 1; k < K; ++k) m = fmax(m, pr.tdf[(size_t)k * C + c]);
  pr.fk[c] = m > -INFINITY ? m : 0.0;
}

__global__ void kblk_weights_kernel(const float* __restrict__ tr, const float* __restrict__ db,
                                    int K, int C, KccPrep pr) {
  const size_t CC = (size_t)C * C, n = (size_t)K * CC;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    const int k = (int)(i / CC), m = (int)((i / C) % C), l = (int)(i % C);
    double f = 0.0, g = 0.0;
    if (k >= 1) {
      const float* tk = tr + (size_t)k * CC;
      f = exp((double)tk[(size_t)m * C + l] + (double)db[(size_t)k * C + l] - pr.fk[l]);
      g = exp((double)tk[(size_t)l * C + m] + (double)db[(size_t)k * C + m] - pr.fk[m]);
    }
    pr.xf[i] = f;
    pr.xb[i] = g;
  }
}

// ---------------------------------------------------------------------------
// Max semiring chain: the same blocks and cluster split, in the log domain
// with (max, +), so no frames are needed:
//   alpha[t,l] = ct[t,l] + max_{s,m} (alpha[s,m] + tr[t-s][m][l] + db[t-s,l] + dt[s,l])
//   beta[s,l]  = max_{u,m} (tr[u-s][l][m] + db[u-s,m] + dt[s,m] + ct[u,m] + beta[u,m])
// pend[j][l] is ct plus the running maximum of row j; the ring holds alpha
// (forward, with dt beside it) or G = ct + beta (backward) of the sources.
template <int P, int CR>
__global__ void __launch_bounds__(kBT, 1) kblkm_chain_kernel(const KccArgs a, int Q) {
  extern __shared__ __align__(16) double bsm[];
  const int C = a.C, K = a.K, T = a.T, kcap = a.kcap;
  const int b = blockIdx.x / Q, rank = blockIdx.x % Q, dir = blockIdx.y, tid = threadIdx.x;
  const bool out0 = rank == 0;
  const int lane = tid & 31, warp = tid >> 5;
  const int Lb = bseq_len(a.lengths, b, T);
  const BlkPlan pl = blk_plan(C, K, P);
  const int NBR = pl.nbr;
  double* ra = bsm + pl.ra;
  double* ry = bsm + pl.ry;
  double* pend = bsm + pl.pend;
  double* part = bsm + pl.part;
  double* ctb = bsm + pl.ctb;
  double* dtb = bsm + pl.dtb;
  double* lv = bsm + pl.lv;
  double* vals = bsm + pl.vals;
  const float* cum_b = a.cum + (size_t)b * (T + 1) * C;
  const float* ps_b = a.ps ? a.ps + (size_t)b * T * C : nullptr;
  const float* pe_b = a.pe ? a.pe + (size_t)b * T * C : nullptr;
  // log weights with the new segment's duration bias: forward rf[k][m][l] =
  // tr[k][m][l] + db[k,l], backward rb[k][m][l] = tr[k][l][m] + db[k,m]
  const double* Wr = dir == 0 ? a.pr.rf : a.pr.rb;
  const size_t CC = (size_t)C * C;
  auto wgt = [&](int k, int m, int l) -> double {
    return (k >= 1 && k <= kcap) ? Wr[(size_t)k * CC + (size_t)m * C + l] : -INFINITY;
  };
  if (dir == 0 && a.ref_ckpt && out0) {
    float* rc = a.ref_ckpt + (size_t)b * a.nref * K * C;
    for (size_t i = tid; i < (size_t)a.nref * K * C; i += kBT)
      rc[i] = (i < (size_t)C) ? 0.f : kRefNegInf;
  }
  __syncthreads();

  const int G = kBT / C, ell = tid % C, sig = tid / C;
  const bool act = sig < G;
  const int nblk = Lb / P + 1;
  const int nnear = (P - 1) * C;
  for (int tau = 0; tau < nblk; ++tau) {
    const int s0 = tau * P, fs = tau % NBR;
    for (int i = tid; i < P * C; i += kBT) {
      const int j = i / C, l = i % C, rho = s0 + j;
      double cv = 0.0, dv = 0.0;
      if (rho <= Lb) {
        const int t = dir == 0 ? rho : Lb - rho;
        const double cu = cum_b[(size_t)t * C + l];
        cv = cu + ((pe_b && t >= 1) ? (double)pe_b[(size_t)(t - 1) * C + l] : 0.0);
        dv = ((ps_b && t < T) ? (double)ps_b[(size_t)t * C + l] : 0.0) - cu;
      }
      ctb[i] = cv;
      dtb[i] = dv;
      // row 0 holds its source values already: alpha = 0, or G = ct + 0
      pend[i] = rho == 0 ? (dir == 0 ? 0.0 : cv) : -INFINITY;
      if (dir == 0) ry[(size_t)(fs * P + j) * C + l] = dv;
    }
    const int bmin = max(0, floor_div(s0 - kcap, P));
    const int nq = tau - bmin;
    __syncthreads();

    // 1. far sums
    if (nq > 0) {
      double out[P];
#pragma unroll
      for (int j = 0; j < P; ++j) out[j] = -INFINITY;
      if (act) {
        const int U = C * nq;
        const int QG = Q * G, slot = rank * G + sig;
        const int u0 = (int)((long long)slot * U / QG), u1 = (int)((long long)(slot + 1) * U / QG);
        double d[2 * P - 1], nx[P];
        int m = u0 / nq, qi = u0 % nq;
        for (int u = u0; u < u1; ++u) {
          if (u > u0 && ++qi == nq) {
            qi = 0;
            ++m;
          }
          const int q = bmin + qi, qs = q % NBR;
          const int D = (tau - q) * P;
          if (u > u0 && qi != 0) {
#pragma unroll
            for (int i = 2 * P - 2; i >= P; --i) d[i] = d[i - P];
#pragma unroll
            for (int i = 0; i < P; ++i) d[i] = nx[i];
          } else {
#pragma unroll
            for (int i = 0; i < 2 * P - 1; ++i) d[i] = wgt(D - P + 1 + i, m, ell);
          }
          if (u + 1 < u1 && qi + 1 < nq) {
#pragma unroll
            for (int i = 0; i < P; ++i) nx[i] = wgt(D - 2 * P + 1 + i, m, ell);
          }
          const int base = qs * P;
          if (dir == 0) {
#pragma unroll
            for (int r = 0; r < P; ++r) {
              const double z = ra[(size_t)(base + r) * C + m] + ry[(size_t)(base + r) * C + ell];
#pragma unroll
              for (int j = 0; j < P; ++j) out[j] = fmax(out[j], d[P - 1 + j - r] + z);
            }
          } else {
            double acc[P];
#pragma unroll
            for (int j = 0; j < P; ++j) acc[j] = -INFINITY;
#pragma unroll
            for (int r = 0; r < P; ++r) {
              const double z = ra[(size_t)(base + r) * C + m];
#pragma unroll
              for (int j = 0; j < P; ++j) acc[j] = fmax(acc[j], d[P - 1 + j - r] + z);
            }
#pragma unroll
            for (int j = 0; j < P; ++j) out[j] = fmax(out[j], acc[j] + dtb[j * C + m]);
          }
        }
      }
#pragma unroll
      for (int j = 0; j < P; ++j) part[j * kBT + tid] = out[j];
      __syncthreads();
      for (int i = tid; i < P * C; i += kBT) {
        const int j = i / C, l = i % C;
        double v = -INFINITY;
        for (int g = 0; g < G; ++g) v = fmax(v, part[j * kBT + g * C + l]);
        if (Q == 1)
          pend[i] = v + ctb[i];
        else
          lv[i] = v;
      }
      if (Q > 1) {
        cg::cluster_group cl = cg::this_cluster();
        cl.sync();
        for (int i = tid; i < P * C; i += kBT) {
          double v = -INFINITY;
          for (int r = 0; r < Q; ++r) v = fmax(v, cl.map_shared_rank(lv, r)[i]);
          pend[i] = v + ctb[i];
        }
        cl.sync();
      } else {
        __syncthreads();
      }
    }

    // 2. the block's rows in order.  pend holds each row's running maximum
    // plus its ct, which is the row's source value once the row is complete
    // (alpha, or G = ct + beta); row j then adds its contributions to rows j + k
    const int last = min(P - 1, Lb - s0);
    auto src = [&](int j, int m) -> double { return pend[j * C + m]; };
    if constexpr (CR > 0) {
      constexpr int NREP = ((P - 1) * CR + kBT - 1) / kBT;
      double w[NREP][CR];
      int kr[NREP], lr[NREP];
      bool vr[NREP];
#pragma unroll
      for (int rep = 0; rep < NREP; ++rep) {
        const int i = tid + rep * kBT;
        kr[rep] = 1 + i / C;
        lr[rep] = i % C;
        vr[rep] = i < nnear && kr[rep] <= kcap;
#pragma unroll
        for (int m = 0; m < CR; ++m)
          w[rep][m] = (vr[rep] && m < C) ? wgt(kr[rep], m, lr[rep]) : -INFINITY;
      }
      for (int j = 0; j <= last; ++j) {
#pragma unroll
        for (int rep = 0; rep < NREP; ++rep) {
          const int jj = j + kr[rep], l = lr[rep];
          if (vr[rep] && jj <= last) {
            double m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
            for (int m = 0; m < CR; ++m)
              if (m < C) {
                const double am = src(j, m) + (dir == 1 ? dtb[jj * C + m] : 0.0);
                m4[m & 3] = fmax(m4[m & 3], am + w[rep][m]);
              }
            const double v = fmax(fmax(m4[0], m4[1]), fmax(m4[2], m4[3])) +
                             (dir == 0 ? dtb[j * C + l] : 0.0) + ctb[jj * C + l];
            pend[jj * C + l] = fmax(pend[jj * C + l], v);
          }
        }
        __syncthreads();
      }
    } else {
      for (int j = 0; j <= last; ++j) {
        for (int i = tid; i < nnear; i += kBT) {
          const int k = 1 + i / C, l = i % C, jj = j + k;
          if (k > kcap || jj > last) continue;
          double v = -INFINITY;
          for (int m = 0; m < C; ++m)
            v = fmax(v, src(j, m) + (dir == 1 ? dtb[jj * C + m] : 0.0) + wgt(k, m, l));
          v += (dir == 0 ? dtb[j * C + l] : 0.0) + ctb[jj * C + l];
          pend[jj * C + l] = fmax(pend[jj * C + l], v);
        }
        __syncthreads();
      }
    }

    // 3. the block's tables, ring rows and row maxima
    const int nrow = last + 1;
    for (int i = tid; i < nrow * C; i += kBT) {
      const int j = i / C, l = i % C, rho = s0 + j;
      const int t = dir == 0 ? rho : Lb - rho;
      ra[(size_t)(fs * P + j) * C + l] = pend[i];
      const double v = rho == 0 ? 0.0 : (dir == 0 ? pend[i] : pend[i] - ctb[i]);
      lv[i] = v;
      if (!out0) continue;
      if (dir == 0) {
        if (a.alpha) a.alpha[((size_t)b * (T + 1) + t) * C + l] = v;
        if (a.ref_ckpt) {
          const int S = a.sref;
          const int ic = (t + S - 1) / S;
          if (ic < a.nref && (long long)ic * S <= Lb && (long long)ic * S - t < K)
            a.ref_ckpt[(((size_t)b * a.nref + ic) * K + (t % K)) * C + l] =
                v > -INFINITY ? (float)v : kRefNegInf;
        }
      } else if (a.beta) {
        a.beta[((size_t)b * (T + 1) + t) * C + l] = v;
      }
    }
    __syncthreads();
    for (int j = warp; j < nrow; j += kBT / 32) {
      double mx = -INFINITY;
      for (int l = lane; l < C; l += 32) mx = fmax(mx, lv[j * C + l]);
      for (int o = 16; o > 0; o >>= 1) mx = fmax(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      if (lane == 0 && dir == 0 && a.amax && out0)
        a.amax[(size_t)b * (T + 1) + (s0 + j)] = mx;
    }
    if (s0 + last == Lb)
      for (int l = tid; l < C; l += kBT) vals[l] = lv[last * C + l];
    __syncthreads();
  }
  if (dir == 0 && tid == 0 && out0) {
    double lz = (double)kRefNegInf;
    if (Lb > 0) {
      double M = -INFINITY;
      for (int q = 0; q < C; ++q) M = fmax(M, vals[q]);
      if (M > -INFINITY) lz = M;
    }
    if (a.logz) a.logz[b] = lz;
    if (a.partition) a.partition[b] = (float)lz;
  }
}

// ---------------------------------------------------------------------------
// Gradients (log semiring).  The segment marginal
//   P(s -> e, m -> l) = exp(alpha[s,m] + tr[e-s][m][l] + db[e-s,l] + dt[s,l] + ct[e,l]
//                           + beta[e,l] - logZ)   (pytorch_reference.py:458-499)
// is written with per-position float64 factors and the weights xf:
//   P = al[s,m] xf[e-s][m][l] Sp[s,l] Ep[e,l] Z(q(s), q(e), l)
//   al = exp(alpha - amax), Sp = exp(st - A[q(s)]), Ep = exp(et + A[q(e)] + fk),
//   Z(q, q') = exp(A[q] - A[q'])
// with st = amax + dt - logZ and et = beta + ct (kcc_terms_kernel) and A[q,l]
// the maximum of st over block q's rows, so Sp <= 1 and the products stay in
// range.  grad_transition[k][m][l] = xf[k][m][l] sum_b g_b sum_s al[s,m] Sp[s,l]
// Ep[s+k,l] Z is a lag correlation per label pair; the start marginal
// Pstart[s,l] = Sp[s,l] sum_{k,m} al[s,m] xf[k][m][l] Ep[s+k,l] Z is a Toeplitz
// product per (source block, label).  Both evaluate P x P register tiles from a
// window of 2P-1 end factors.

// A[b][q][l]: maximum of st over the rows s < len of block q; a block without a
// finite one takes -max(et + fk) of its rows (0 when none), which keeps its end
// factors at most 1
__global__ void kblk_anchor_kernel(const KccArgs a) {
  const int C = a.C, T = a.T, nb = T / kBP + 1;
  const size_t n = (size_t)a.B * nb * C;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    const int c = (int)(i % C);
    const size_t bq = i / C;
    const int q = (int)(bq % nb), b = (int)(bq / nb);
    const int Lb = bseq_len(a.lengths, b, T);
    const size_t row0 = (size_t)b * (T + 1);
    double m = -INFINITY, me = -INFINITY;
    for (int r = 0; r < kBP; ++r) {
      const int s = q * kBP + r;
      if (s < Lb) m = fmax(m, a.st[(row0 + s) * C + c]);
      if (s >= 1 && s <= Lb) me = fmax(me, a.et[(row0 + s) * C + c]);
    }
    a.anc[i] = m > -INFINITY ? m : (me > -INFINITY ? -(me + a.pr.fk[c]) : 0.0);
    if (i == 0 && a.kflag) *a.kflag = 0;  // kblk_factor_kernel sets it
  }
}

// al, and st / et replaced by Sp / Ep in place
__global__ void kblk_factor_kernel(const KccArgs a) {
  const int C = a.C, T = a.T, nb = T / kBP + 1;
  const size_t n = (size_t)a.B * (T + 1) * C;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    const int c = (int)(i % C);
    const size_t bt = i / C;
    const int t = (int)(bt % (T + 1)), b = (int)(bt / (T + 1));
    const int Lb = bseq_len(a.lengths, b, T);
    const double A = a.anc[((size_t)b * nb + t / kBP) * C + c];
    const double A1 = t >= kBP ? a.anc[((size_t)b * nb + t / kBP - 1) * C + c] : 0.0;
    double av = 0.0, sv = 0.0, ev = 0.0, ev1 = 0.0;
    if (t < Lb) {
      const double nm = a.amax[bt], x = a.alpha[i];
      if (nm > -INFINITY && x > -INFINITY) av = exp(x - nm);
      const double st = a.st[i];
      if (st > -INFINITY) sv = exp(st - A);
    }
    if (t >= 1 && t <= Lb) {
      const double et = a.et[i];
      if (et > -INFINITY) {
        const double x0 = et + A + a.pr.fk[c], x1 = et + A1 + a.pr.fk[c];
        // near the float64 range the block factoring loses terms: the gradients
        // are redone per item in the log domain (launch_kcc_grads)
        if (a.kflag && (x0 > 600.0 || (t >= kBP && x1 > 600.0))) *a.kflag = 1;
        ev = exp(fmin(x0, 700.0));
        if (t >= kBP) ev1 = exp(fmin(x1, 700.0));
      }
    }
    a.al[i] = av;
    a.st[i] = sv;
    a.et[i] = ev;
    a.ep1[i] = ev1;
  }
}

// the window of end factors for source block q and lag chunk lam: rows
// (q + lam) * P + x, x < 2P-1, relative to block q's anchor
template <int P>
__device__ __forceinline__ void end_window(const KccArgs& a, const double* anc, size_t row0,
                                           int Lb, int nb, int q, int lam, int l, double* w) {
  const int C = a.C, q1 = q + lam;
  const double Aq = anc[(size_t)q * C + l];
  const double z1 = q1 < nb ? exp(fmin(Aq - anc[(size_t)q1 * C + l], 700.0)) : 0.0;
  const double z2 = q1 + 1 < nb ? exp(fmin(Aq - anc[(size_t)(q1 + 1) * C + l], 700.0)) : 0.0;
#pragma unroll
  for (int x = 0; x < 2 * P - 1; ++x) {
    const int e = q1 * P + x;
    w[x] = e <= Lb ? a.et[(row0 + e) * C + l] * (x < P ? z1 : z2) : 0.0;
  }
}

__device__ __forceinline__ void cp_async8z(double* dst, const double* src, bool valid) {
  const unsigned d = (unsigned)__cvta_generic_to_shared(dst);
  const int n = valid ? 8 : 0;  // 0: the destination is zero-filled
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;\n" ::"r"(d), "l"(src), "r"(n)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit_g() {
  asm volatile("cp.async.commit_group;\n" ::: "memory");
}
__device__ __forceinline__ void cp_async_wait_1() {
  asm volatile("cp.async.wait_group 1;\n" ::: "memory");
}

// part[slice][m][(k-1)*C + l] = sum over the slice's sequences and sources of
// g_b al[s,m] Sp[s,l] Ep[s+k,l] Z.  A CTA takes one lag chunk lam (k = lam*P + i),
// one slice and up to blockDim label pairs; its items are the (sequence, source
// block q) of the slice (a class of sequences, and a chunk of their source
// blocks when there are more slices than sequences).  An item's rows -- al and Sp of the block's sources,
// the end factors of rows (q+lam)*P .. +2P-2 (block q+lam relative to its own
// anchor, block q+lam+1 relative to block q+lam's) and the two anchors -- are
// staged in shared memory by cp.async, one item ahead, so the item's factor
// exp(A[q] - A[q+lam]) is a single scale of the source values.
template <int P>
__global__ void __launch_bounds__(kBT, 2) kblk_tr_kernel(const KccArgs a, int nch, int npg) {
  extern __shared__ __align__(16) double tsm[];
  const int C = a.C, T = a.T, kcap = a.kcap, nb = T / P + 1;
  const int npair = C * C, tid = threadIdx.x, nt = blockDim.x;
  const int pg = blockIdx.x % npg, rest = blockIdx.x / npg;
  const int lam = rest % nch, slice = rest / nch;
  const int pair = pg * nt + tid;
  const bool act = pair < npair;
  const int m = act ? pair / C : 0, l = act ? pair % C : 0;
  constexpr int RW = 4 * P - 1;  // staged rows: al (P), Sp (P), end factors (2P-1)
  const int SZ = (RW + 2) * C;   // and the two anchor rows
  double* buf0 = tsm;
  double* buf1 = tsm + SZ;
  auto nq_of = [&](int b) -> int {
    const int Lb = bseq_len(a.lengths, b, T);
    if (Lb <= 0 || a.grad_output[b] == 0.0f) return 0;
    const int n = min((Lb - 1) / P + 1, Lb / P - lam + 1);
    return n > 0 ? n : 0;
  };
  // slice = (sequence class bs, source-block chunk qc): sequences bs, bs + nbs, ...
  // and, of each, the qc-th of nqc equal chunks of its source blocks
  const int nbs = min(a.B, a.nslice), nqc = a.nslice / nbs;
  const int bs = slice % nbs, qc = slice / nbs;
  auto q_hi = [&](int b) -> int {
    const int nq = nq_of(b), ql = (nq + nqc - 1) / nqc;
    return min(nq, (qc + 1) * ql);
  };
  auto first_from = [&](int b0, int& b, int& q) -> bool {
    for (b = b0; b < a.B; b += nbs) {
      const int nq = nq_of(b), ql = (nq + nqc - 1) / nqc;
      if (qc * ql < min(nq, (qc + 1) * ql)) {
        q = qc * ql;
        return true;
      }
    }
    return false;
  };
  // this thread's staged elements i = tid + j * nt as (row x, label c), advanced
  // without divisions
  const int x0 = tid / C, c0 = tid % C, dx = nt / C, dc = nt % C;
  auto stage = [&](int b, int q, double* d) {
    const int Lb = bseq_len(a.lengths, b, T);
    const size_t row0 = (size_t)b * (T + 1);
    int x = x0, c = c0;
    for (int i = tid; i < RW * C; i += nt) {
      const double* src = a.al;
      bool ok = false;
      if (x < P) {
        const int s = q * P + x;
        ok = s < Lb;
        if (ok) src = a.al + (row0 + s) * C + c;
      } else if (x < 2 * P) {
        const int s = q * P + x - P;
        ok = s < Lb;
        if (ok) src = a.st + (row0 + s) * C + c;
      } else {
        const int xx = x - 2 * P, e = (q + lam) * P + xx;
        ok = e <= Lb;
        if (ok) src = (xx < P ? a.et : a.ep1) + (row0 + e) * C + c;
      }
      cp_async8z(d + i, src, ok);
      x += dx;
      c += dc;
      if (c >= C) {
        c -= C;
        ++x;
      }
    }
    for (int i = tid; i < 2 * C; i += nt) {
      const int qq = i < C ? q : q + lam;
      cp_async8z(d + RW * C + i, a.anc + ((size_t)b * nb + qq) * C + (i % C), true);
    }
  };
  double acc[P];
#pragma unroll
  for (int i = 0; i < P; ++i) acc[i] = 0.0;
  int b = 0, q = 0, n = 0;
  bool have = first_from(bs, b, q);
  if (have) stage(b, q, buf0);
  cp_async_commit_g();
  while (have) {
    int bn = b, qn = q;
    bool more;
    if (q + 1 < q_hi(b)) {
      qn = q + 1;
      more = true;
    } else {
      more = first_from(b + nbs, bn, qn);
    }
    if (more) stage(bn, qn, (n & 1) ? buf0 : buf1);
    cp_async_commit_g();
    cp_async_wait_1();
    __syncthreads();
    const double* d = (n & 1) ? buf1 : buf0;
    if (act) {
      const double z = (double)a.grad_output[b] *
                       exp(fmin(d[RW * C + l] - d[(RW + 1) * C + l], 700.0));
      double w[2 * P - 1];
#pragma unroll
      for (int x = 0; x < 2 * P - 1; ++x) w[x] = d[(2 * P + x) * C + l];
#pragma unroll
      for (int r = 0; r < P; ++r) {
        const double u = z * d[r * C + m] * d[(P + r) * C + l];
#pragma unroll
        for (int i = 0; i < P; ++i) acc[i] = fma(u, w[r + i], acc[i]);
      }
    }
    __syncthreads();  // this buffer is staged again two items later
    b = bn;
    q = qn;
    have = more;
    ++n;
  }
  if (!act) return;
  const int ncol = kcap * C;
  double* out = a.part_tr + (size_t)slice * C * ncol + (size_t)m * ncol;
#pragma unroll
  for (int i = 0; i < P; ++i) {
    const int k = lam * P + i;
    if (k >= 1 && k <= kcap) out[(size_t)(k - 1) * C + l] = acc[i];
  }
}

// max semiring: the end marginal of every (position, label), summed over its
// incoming segments, Pend[e,l] = Ep[e,l] sum_{s,m} al[s,m] xf[e-s][m][l] Sp[s,l] Z
// (the log semiring has it as exp(alpha + beta - logZ)).  Thread (sequence,
// target block tau, label l): for each source block q within reach and source
// label m, the P x P Toeplitz tile out[j] += sum_r x[D + j - r][m][l] z[r] from a
// window of 2P-1 weights, as in the chain's far sums.
template <int P>
__global__ void __launch_bounds__(kBT, 1) kblk_pend_kernel(const KccArgs a) {
  const int C = a.C, T = a.T, kcap = a.kcap, nb = T / P + 1;
  const long long gid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const int l = (int)(gid % C);
  const long long rest = gid / C;
  const int tau = (int)(rest % nb), b = (int)(rest / nb);
  if (b >= a.B) return;
  const int Lb = bseq_len(a.lengths, b, T);
  const size_t row0 = (size_t)b * (T + 1);
  const double* anc = a.anc + (size_t)b * nb * C;
  const size_t CC = (size_t)C * C;
  const int e0 = tau * P;
  double out[P];
#pragma unroll
  for (int j = 0; j < P; ++j) out[j] = 0.0;
  if (e0 <= Lb) {
    const double At = anc[(size_t)tau * C + l];
    const int qlo = max(0, floor_div(e0 - kcap, P));
    for (int q = qlo; q <= tau; ++q) {
      const int D = (tau - q) * P;
      const double Z = exp(fmin(anc[(size_t)q * C + l] - At, 700.0));
      double zs[P];
#pragma unroll
      for (int r = 0; r < P; ++r) {
        const int s = q * P + r;
        zs[r] = s < Lb ? a.st[(row0 + s) * C + l] * Z : 0.0;
      }
      for (int m = 0; m < C; ++m) {
        double d[2 * P - 1];
#pragma unroll
        for (int i = 0; i < 2 * P - 1; ++i) {
          const int k = D - P + 1 + i;
          d[i] = (k >= 1 && k <= kcap) ? __ldg(a.pr.xf + (size_t)k * CC + (size_t)m * C + l) : 0.0;
        }
#pragma unroll
        for (int r = 0; r < P; ++r) {
          const int s = q * P + r;
          const double z = s < Lb ? a.al[(row0 + s) * C + m] * zs[r] : 0.0;
#pragma unroll
          for (int j = 0; j < P; ++j) out[j] = fma(d[P - 1 + j - r], z, out[j]);
        }
      }
    }
  }
#pragma unroll
  for (int j = 0; j < P; ++j) {
    const int e = e0 + j;
    if (e > T) break;
    const size_t i = (row0 + e) * C + l;
    a.pend[i] = (e >= 1 && e <= Lb) ? a.et[i] * out[j] : 0.0;
  }
}

// start marginals and the position gradients; thread (sequence, source block,
// label) for every row 0 .. T
template <int P>
__global__ void __launch_bounds__(kBT, 1) kblk_pos_kernel(const KccArgs a, int nch) {
  const int C = a.C, T = a.T, kcap = a.kcap, nb = T / P + 1;
  const long long gid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const int l = (int)(gid % C);
  const long long rest = gid / C;
  const int q = (int)(rest % nb), b = (int)(rest / nb);
  if (b >= a.B) return;
  const int Lb = bseq_len(a.lengths, b, T);
  const size_t row0 = (size_t)b * (T + 1);
  const double* anc = a.anc + (size_t)b * nb * C;
  const size_t CC = (size_t)C * C;
  const int s0 = q * P;
  double out[P];
#pragma unroll
  for (int r = 0; r < P; ++r) out[r] = 0.0;
  if (s0 < Lb) {
    for (int lam = 0; lam < nch && (q + lam) * P <= Lb; ++lam) {
      double w[2 * P - 1];
      end_window<P>(a, anc, row0, Lb, nb, q, lam, l, w);
      for (int m = 0; m < C; ++m) {
        double xk[P], V[P];
#pragma unroll
        for (int i = 0; i < P; ++i) {
          const int k = lam * P + i;
          xk[i] = (k >= 1 && k <= kcap) ? __ldg(a.pr.xf + (size_t)k * CC + (size_t)m * C + l) : 0.0;
          V[i] = 0.0;
        }
#pragma unroll
        for (int i = 0; i < P; ++i)
#pragma unroll
          for (int r = 0; r < P; ++r) V[r] = fma(xk[i], w[r + i], V[r]);
#pragma unroll
        for (int r = 0; r < P; ++r) {
          const int s = s0 + r;
          const double av = s < Lb ? a.al[(row0 + s) * C + m] : 0.0;
          out[r] = fma(av, V[r], out[r]);
        }
      }
    }
  }
  const double g = (double)a.grad_output[b];
  const double lz = a.logz[b];
#pragma unroll
  for (int r = 0; r < P; ++r) {
    const int s = s0 + r;
    if (s > T) break;
    const size_t i = (row0 + s) * C + l;
    double pend = 0.0;
    if (s >= 1 && s <= Lb) {
      if (a.semiring == SEMICRF_MAX) {
        pend = a.pend[i];
      } else {
        const double v = a.alpha[i] + a.beta[i] - lz;
        pend = v > -INFINITY ? exp(v) : 0.0;
      }
    }
    const double pst = s < Lb ? a.st[i] * out[r] : 0.0;
    a.grad_cum[i] = (float)(g * (pend - pst));
    if (a.grad_ps && s < T) a.grad_ps[((size_t)b * T + s) * C + l] = (float)(g * pst);
    if (a.grad_pe && s >= 1) a.grad_pe[((size_t)b * T + s - 1) * C + l] = (float)(g * pend);
  }
}

}  // namespace

bool kblk_supported(int C, int K) {
  if (K < 2 || C < 1 || C > 128) return false;
  return blk_plan(C, K, kBP).total * 8 <= kBSmemMax;
}

cudaError_t launch_kblk_prep(const float* tr, const float* db, int K, int C, const KccPrep& pr,
                             cudaStream_t s) {
  if (!pr.xf) return cudaSuccess;
  kblk_fk_kernel<<<(C + 127) / 128, 128, 0, s>>>(K, C, pr);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const size_t n = (size_t)K * C * C;
  size_t g = (n + 255) / 256;
  if (g > device_sm_count() * 8) g = device_sm_count() * 8;
  kblk_weights_kernel<<<(int)(g < 1 ? 1 : g), 256, 0, s>>>(tr, db, K, C, pr);
  return cudaGetLastError();
}

cudaError_t launch_kblk_chains(const KccArgs& a, int ndir, cudaStream_t s) {
  if (a.B <= 0) return cudaSuccess;
  const size_t bytes = blk_plan(a.C, a.K, kBP).total * 8;
  auto go = [&](auto kern) -> cudaError_t {
    cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e != cudaSuccess) return e;
    // a cluster of Q CTAs per chain when the chains alone leave SMs idle and
    // all the clusters fit at once
    const int nsm = device_sm_count();
    const int nchain = a.B * ndir;
    for (int Q = kBMaxQ; Q >= 2; Q /= 2) {
      if (nchain * Q > nsm) continue;
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(a.B * Q, ndir);
      cfg.blockDim = dim3(kBT);
      cfg.dynamicSmemBytes = bytes;
      cfg.stream = s;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = Q;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      int ncl = 0;
      if (cudaOccupancyMaxActiveClusters(&ncl, kern, &cfg) != cudaSuccess) {
        cudaGetLastError();
        continue;
      }
      if (ncl < nchain) continue;
      return cudaLaunchKernelEx(&cfg, kern, a, Q);
    }
    kern<<<dim3(a.B, ndir), kBT, bytes, s>>>(a, 1);
    return cudaGetLastError();
  };
  // register-held in-block weights for C <= kRegC, sized to the next multiple of 8
  if (a.semiring == SEMICRF_MAX) {
    if (a.C <= 8) return go(kblkm_chain_kernel<kBP, 8>);
    if (a.C <= 16) return go(kblkm_chain_kernel<kBP, 16>);
    if (a.C <= 24) return go(kblkm_chain_kernel<kBP, 24>);
    if (a.C <= kRegC) return go(kblkm_chain_kernel<kBP, kRegC>);
    return go(kblkm_chain_kernel<kBP, 0>);
  }
  if (a.C <= 8) return go(kblk_chain_kernel<kBP, 8>);
  if (a.C <= 16) return go(kblk_chain_kernel<kBP, 16>);
  if (a.C <= 24) return go(kblk_chain_kernel<kBP, 24>);
  if (a.C <= kRegC) return go(kblk_chain_kernel<kBP, kRegC>);
  return go(kblk_chain_kernel<kBP, 0>);
}

size_t kblk_anchor_rows(int T) { return (size_t)(T / kBP + 1); }

// label pairs per CTA of the transition-gradient kernel: npg CTAs of tpb threads
static void tr_shape(int C, int& npg, int& tpb) {
  const int npair = C * C;
  npg = (npair + kBT - 1) / kBT;
  tpb = ((npair + npg - 1) / npg + 31) / 32 * 32;
}

int kblk_tr_slices(int B, int K, int C) {
  int npg, tpb;
  tr_shape(C, npg, tpb);
  const long long per = (long long)npg * ((K + kBP - 1) / kBP);  // CTAs per slice
  const long long want = device_sm_count() * 2LL * 4;                        // four waves of two CTAs per SM
  long long ns = (want + per - 1) / per;
  if (ns < 1) ns = 1;
  // slices cover sequences first, then chunks of each sequence's source blocks
  const long long nbs = ns < B ? ns : (B > 0 ? B : 1);
  return (int)(nbs * (ns / nbs));
}

cudaError_t launch_kblk_grads(const KccArgs& a, cudaStream_t s) {
  const int nb = a.T / kBP + 1;
  auto grid = [](size_t n, int t) {
    size_t g = (n + t - 1) / t;
    const size_t gmax = (size_t)device_sm_count() * 16;
    if (g > gmax) g = gmax;
    return (int)(g < 1 ? 1 : g);
  };
  kblk_anchor_kernel<<<grid((size_t)a.B * nb * a.C, 256), 256, 0, s>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  kblk_factor_kernel<<<grid((size_t)a.B * (a.T + 1) * a.C, 256), 256, 0, s>>>(a);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const int nch = (a.K + kBP - 1) / kBP;  // lag chunks covering k = 0 .. K-1
  const long long npos = (long long)a.B * nb * a.C;
  if (a.semiring == SEMICRF_MAX) {
    kblk_pend_kernel<kBP><<<(unsigned)((npos + kBT - 1) / kBT), kBT, 0, s>>>(a);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  kblk_pos_kernel<kBP><<<(unsigned)((npos + kBT - 1) / kBT), kBT, 0, s>>>(a, nch);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  int npg, tpb;
  tr_shape(a.C, npg, tpb);
  const size_t tbytes = (size_t)2 * (4 * kBP - 1 + 2) * a.C * 8;
  e = cudaFuncSetAttribute(kblk_tr_kernel<kBP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)tbytes);
  if (e != cudaSuccess) return e;
  kblk_tr_kernel<kBP><<<npg * nch * a.nslice, tpb, tbytes, s>>>(a, nch, npg);
  return cudaGetLastError();
}

}  // namespace semicrf
