// lchain_cl.cu -- float64 log-semiring chains for large label sets
// (64 < C <= 256) on thread-block clusters of four CTAs.
//
// Same recurrence, linear-domain formulation and output tables as the
// generic chain (lchain.cu; reference semantics streaming/pytorch_reference.py:
// 116-273 forward and the beta recursion of :276-525):
//     a[u,c]  = g[u,c] * sum_k E[u-k,c] * Db[k,c]
//     ym[u,c] = sum_c' a[u,c'] * Mx[c',c]
//     E[u,c]  = ym[u,c] * h[u,c]
// At large C the per-position cost is the mat-vec: one CTA would stream the
// whole C x C float64 factor Mx (512 KB at C = 256) from L2 every position.
// Here CTA r of the cluster owns labels [r*CL, r*CL + CL), CL = ceil(C/4):
// its column slice of Mx (C x CL doubles, 128 KB at C = 256) is spread over
// the registers of its 512 threads (at most 32 doubles each: thread (o, p)
// holds Mx[q][o] for its input slice p), and its labels' source ring, duration
// factors, far sums and g/h factors are in shared memory.
//
// A cluster runs G chains of the same direction side by side (G = 2 when the
// batch allows): the register slice of Mx serves every chain's mat-vec, and
// one cluster barrier per position serves all G.  Per position each CTA
// computes a[u,c] of its labels for each chain, stores them into all four
// CTAs' shared memory (distributed shared memory), and after the barrier
// every CTA holds each chain's full vector a[u,.] and forms its slice of the
// mat-vecs.  Block normalisers and log Z are read off the same vectors.  The
// state vectors are double-buffered, so the one barrier per position also
// orders their reuse.  Chains of different lengths run to the longest; a
// chain past its end computes nothing and writes nothing.
//
// Whole chains only (mode 0): no reference ring-checkpoint output and no
// restart records; those run on lchain.cu.  The tables written (a, A, n per
// position) are identical in meaning to lchain.cu's, so lmarg.cu derives the
// gradients unchanged.

#include <cooperative_groups.h>

#include <cstdlib>

#include "semicrf_internal.cuh"

namespace semicrf {

namespace {

namespace cg = cooperative_groups;

constexpr int kNT = 512;
constexpr int kNCL = 4;  // CTAs per cluster
constexpr int kMQ = 32;  // most Mx inputs one thread holds (C <= 256)
constexpr int kLP = 4;   // targets per block
constexpr size_t kSmemMax = 227 * 1024;
constexpr double kHi = 1e78, kLo = 1e-78;  // re-anchor when the newest source leaves this

struct CPlan {
  int C, CL, CPAD, K, kcap, R, kx, nparts, qper, nsplit, G;
  bool db_smem;
  // offsets in doubles; per-chain arrays repeat G times with the given stride
  int o_ring, o_abuf, o_ypart, o_g, o_h, o_far, o_part, o_pcu, o_pto, o_pso, o_dbe, o_dbmax,
      o_colmax, o_ref, o_fac, o_flag, o_misc, total;
};

__host__ __device__ inline void cmake(CPlan& p, int C, int K, int G, bool db_smem) {
  p.C = C;
  p.G = G;
  p.CL = (C + kNCL - 1) / kNCL;
  p.K = K;
  p.kcap = K > 1 ? K - 1 : 1;
  p.R = p.kcap + kLP;
  p.kx = p.kcap + kPrepRowsExtra;
  p.nparts = kNT / p.CL;
  p.qper = (C + p.nparts - 1) / p.nparts;
  p.nsplit = kNT / (G * p.CL);  // far-sum splits per (chain, label)
  if (p.nsplit < 1) p.nsplit = 1;
  // state vector length: the mat-vec reads inputs in groups of four up to
  // nparts * qper; entries past C stay zero
  {
    const int span = p.nparts * p.qper > C ? p.nparts * p.qper : C;
    p.CPAD = (span + 4 + 1) & ~1;
  }
  p.db_smem = db_smem;
  int o = 0;
  auto take = [&](int n) {
    const int r = o;
    o += (n + 1) & ~1;  // keep 16-byte alignment
    return r;
  };
  const int CL = p.CL;
  p.o_ring = take(G * p.R * CL);
  p.o_abuf = take(2 * G * p.CPAD);  // [parity][chain][CPAD]
  p.o_ypart = take(G * p.nparts * CL);
  p.o_g = take(G * kLP * CL);
  p.o_h = take(G * kLP * CL);
  p.o_far = take(G * kLP * CL);
  p.o_part = take(G * p.nsplit * kLP * CL);
  p.o_pcu = take(G * kLP * CL);
  p.o_pto = take(G * kLP * CL);
  p.o_pso = take(G * kLP * CL);
  p.o_dbe = db_smem ? take(p.kx * CL) : -1;
  p.o_dbmax = take(CL);
  p.o_colmax = take(CL);
  p.o_ref = take(G * CL);
  p.o_fac = take(G * CL);
  p.o_flag = take(G * CL);  // ints, one double each
  p.o_misc = take(16 * G);
  p.total = o;
}

__host__ __device__ inline bool cchoose(CPlan& p, int C, int K, int G) {
  cmake(p, C, K, G, true);
  if ((size_t)p.total * 8 <= kSmemMax) return true;
  cmake(p, C, K, G, false);
  return (size_t)p.total * 8 <= kSmemMax;
}

template <int G>
__global__ void __cluster_dims__(kNCL, 1, 1) __launch_bounds__(kNT, 1)
    lchain_cl_kernel(const __grid_constant__ LChainLaunch L, int ngroups) {
  extern __shared__ __align__(16) double csm[];
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // cluster -> (role, group of G chains of that role)
  const int cid = (int)blockIdx.x / kNCL;
  const bool role1 = cid >= ngroups;
  const LChainArgs& A = role1 ? L.a1 : L.a0;
  const int grp = role1 ? cid - ngroups : cid;
  const int C = L.C, K = L.K, T = L.T;
  const int dir = A.dir;
  const double csign = dir == 0 ? 1.0 : -1.0;
  int bq[G], Lq[G];
  int Lmax = 0;
#pragma unroll
  for (int g = 0; g < G; ++g) {
    bq[g] = grp * G + g;
    int l = 0;
    if (bq[g] < L.B) {
      const long long lraw = A.lengths[bq[g]];
      l = lraw < 0 ? 0 : (lraw > T ? T : (int)lraw);
    }
    Lq[g] = l;
    Lmax = Lmax > l ? Lmax : l;
  }

  CPlan pl;
  cchoose(pl, C, K, G);
  const int CL = pl.CL, kcap = pl.kcap, R = pl.R;
  const int c0 = rank * CL;
  const int Cr = C - c0 < CL ? (C - c0 > 0 ? C - c0 : 0) : CL;  // labels of this CTA
  double* ring0 = csm + pl.o_ring;     // [G][R][CL]
  double* abuf = csm + pl.o_abuf;      // [2][G][CPAD]
  double* ypart = csm + pl.o_ypart;    // [G][nparts][CL]
  double* gf0 = csm + pl.o_g;          // [G][kLP][CL]
  double* hf0 = csm + pl.o_h;
  double* far0 = csm + pl.o_far;
  double* part0 = csm + pl.o_part;     // [G][nsplit][kLP][CL]
  double* pcu0 = csm + pl.o_pcu;
  double* pto0 = csm + pl.o_pto;
  double* pso0 = csm + pl.o_pso;
  double* dbes = pl.db_smem ? csm + pl.o_dbe : nullptr;
  double* dbmax = csm + pl.o_dbmax;
  double* colmax = csm + pl.o_colmax;
  double* ref0 = csm + pl.o_ref;       // [G][CL]
  double* fac0 = csm + pl.o_fac;
  int* flag0 = reinterpret_cast<int*>(csm + pl.o_flag);  // [G][2 CL]
  double* misc0 = csm + pl.o_misc;     // [G][16]
  int* anyflag = reinterpret_cast<int*>(misc0 + 5);  // one flag for all chains
  const int RB = R * CL, PB = kLP * CL;

  auto abv = [&](int par, int g) { return abuf + (size_t)(par * G + g) * pl.CPAD; };
  auto cpos = [&](int g, int u) { return dir == 0 ? u : Lq[g] - u; };
  auto cum_of = [&](int g) { return A.cum + (size_t)bq[g] * (T + 1) * C; };
  // offsets and cum of global label gc of chain g at chain position u
  auto soff_at = [&](int g, int u, int gc) -> double {
    const int t = cpos(g, u);
    if (dir == 0)
      return (A.ps && t < T) ? (double)A.ps[((size_t)bq[g] * T + t) * C + gc] : 0.0;
    return (A.pe && t >= 1) ? (double)A.pe[((size_t)bq[g] * T + t - 1) * C + gc] : 0.0;
  };
  auto toff_at = [&](int g, int u, int gc) -> double {
    const int t = cpos(g, u);
    if (dir == 0)
      return (A.pe && t >= 1) ? (double)A.pe[((size_t)bq[g] * T + t - 1) * C + gc] : 0.0;
    return (A.ps && t < T) ? (double)A.ps[((size_t)bq[g] * T + t) * C + gc] : 0.0;
  };
  auto cumd = [&](int g, int u, int gc) -> double {
    return (double)cum_of(g)[(size_t)cpos(g, u) * C + gc];
  };
  auto dbe_at = [&](int k, int i) -> double {
    return pl.db_smem ? dbes[k * CL + i] : L.dbe[(size_t)k * C + c0 + i];
  };

  // ---- constants ----------------------------------------------------------
  if (tid == 0) anyflag[0] = 0;
  for (int i = tid; i < 2 * G * pl.CPAD; i += kNT) abuf[i] = 0.0;
  for (int i = tid; i < CL; i += kNT) {
    dbmax[i] = i < Cr ? (double)L.dbmax[c0 + i] : 0.0;
    colmax[i] = i < Cr ? (double)A.colmax[c0 + i] : 0.0;
  }
  for (int i = tid; i < G * CL; i += kNT) flag0[2 * i] = 0;
  if (pl.db_smem)
    for (int i = tid; i < pl.kx * CL; i += kNT) {
      const int k = i / CL, o = i % CL;
      dbes[i] = o < Cr ? L.dbe[(size_t)k * C + c0 + o] : 0.0;
    }
  __syncthreads();

  // label threads: (chain gs, label c); the other threads help in the
  // parallel phases only
  const int gs = tid / CL, c = tid % CL;
  const bool lt = gs < G;           // a label thread
  const bool cv = lt && c < Cr;     // ... of a label this CTA owns
  const int gcl = c0 + c;
  double dbj[kLP + 1];
#pragma unroll
  for (int j = 0; j <= kLP; ++j) dbj[j] = (cv && j >= 1) ? dbe_at(j, c) : 0.0;
  const double ecol = cv ? exp(colmax[c]) : 0.0;
  double* ring_me = ring0 + (size_t)(lt ? gs : 0) * RB;
  double* atab_me = (lt && A.a_tab) ? A.a_tab + (size_t)bq[gs] * (T + 1) * C : nullptr;
  double* Atab_me = (lt && A.A_tab) ? A.A_tab + (size_t)bq[gs] * (T + 1) * C : nullptr;

  // this thread's part of the Mx slice: inputs q0 + j, j < kMQ, of label o
  const int mo = tid % CL, mp = tid / CL;
  const int mq0 = mp * pl.qper;
  double mr[kMQ];
#pragma unroll
  for (int j = 0; j < kMQ; ++j) {
    const int q = mq0 + j;
    mr[j] = (mp < pl.nparts && mo < Cr && j < pl.qper && q < C) ? A.mx[(size_t)q * C + c0 + mo]
                                                                 : 0.0;
  }
  // ym of every chain for this CTA's labels from the full state vectors in
  // buffer par: every thread sums its slice of the inputs for one label, then
  // the label thread of (chain, label) adds the slices
  auto matvec = [&](int par) -> double {
    if (mp < pl.nparts) {
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const double* av = abv(par, g);
        double y0 = 0.0, y1 = 0.0, y2 = 0.0, y3 = 0.0;
#pragma unroll
        for (int j = 0; j < kMQ; j += 4) {
          if (j < pl.qper) {
            // inputs past C (or past this slice) meet zero registers; av is
            // padded to the slice grid so these reads stay inside abuf
            y0 = fma(av[mq0 + j], mr[j], y0);
            y1 = fma(av[mq0 + j + 1], mr[j + 1], y1);
            y2 = fma(av[mq0 + j + 2], mr[j + 2], y2);
            y3 = fma(av[mq0 + j + 3], mr[j + 3], y3);
          }
        }
        ypart[(g * pl.nparts + mp) * CL + mo] = (y0 + y1) + (y2 + y3);
      }
    }
    __syncthreads();
    double ym = 0.0;
    if (lt)
      for (int p = 0; p < pl.nparts; ++p) ym += ypart[(gs * pl.nparts + p) * CL + c];
    return ym;
  };
  // store the active label threads' a values into buffer par of every CTA of
  // the cluster, then wait until all four CTAs have done so.  A chain past its
  // end stores nothing, so its buffers keep its last state (log Z reads it).
  auto publish = [&](double a, int par, bool on) {
    if (on) {
#pragma unroll
      for (int r = 0; r < kNCL; ++r) {
        double* dst = cluster.map_shared_rank(abv(par, gs), r);
        dst[gcl] = a;
      }
    }
    cluster.sync();
  };
  // max and sum over a full state vector (one warp)
  auto vec_max = [&](const double* av) -> double {
    double m = 0.0;
    for (int q = lane; q < C; q += 32) m = fmax(m, av[q]);
    for (int o = 16; o > 0; o >>= 1) m = fmax(m, __shfl_xor_sync(0xffffffffu, m, o));
    return m;
  };
  auto vec_sum = [&](const double* av) -> double {
    double s = 0.0;
    for (int q = lane; q < C; q += 32) s += av[q];
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    return s;
  };

  // ---- initial state ------------------------------------------------------
  {
    double a0 = 0.0, ym0 = 0.0;
    if (dir == 0) {
      // alpha[0] = 0 for every label, n = 0: the full vectors are known locally
      for (int i = tid; i < G * C; i += kNT) abv(0, i / C)[i % C] = 1.0;
      __syncthreads();
      a0 = cv ? 1.0 : 0.0;
      ym0 = matvec(0);
      __syncthreads();
      for (int i = tid; i < G * C; i += kNT) abv(0, i / C)[i % C] = 0.0;
    } else {
      ym0 = cv ? exp(-colmax[c]) : 0.0;  // beta[L] = 0
    }
    if (cv) {
      // a padding chain of an odd batch (index >= B) reads no input
      const bool real = bq[gs] < L.B;
      const double so = real ? soff_at(gs, 0, gcl) : 0.0;
      const double cu = real ? cumd(gs, 0, gcl) : 0.0;
      ref0[gs * CL + c] = (ym0 > 0.0) ? log(ym0) + colmax[c] + so - csign * cu : 0.0;
      ring_me[0 * CL + c] = (ym0 > 0.0) ? 1.0 : 0.0;
      if (real) {
        const int t0 = cpos(gs, 0);
        if (atab_me) atab_me[(size_t)t0 * C + gcl] = a0;
        if (Atab_me) Atab_me[(size_t)t0 * C + gcl] = ym0 * ecol;
      }
    }
    if (tid < G) {
      misc0[tid * 16 + 0] = 0.0;  // n of position 0
      misc0[tid * 16 + 1] = 0.0;  // n of the first block: log max a[0] = 0 (alpha) or 0 (beta)
      if (rank == 0 && bq[tid] < L.B && A.n_tab)
        A.n_tab[(size_t)bq[tid] * (T + 1) + cpos(tid, 0)] = 0.0;
    }
  }
  // every CTA's constants are in place before any remote store reaches it
  cluster.sync();

  // element g of a per-chain register array, by selects over the unrolled index
  auto pick_i = [&](const int (&v)[G], int g) -> int {
    int r = v[0];
#pragma unroll
    for (int q = 1; q < G; ++q)
      if (q == g) r = v[q];
    return r;
  };
  auto pick_d = [&](const double (&v)[G], int g) -> double {
    double r = v[0];
#pragma unroll
    for (int q = 1; q < G; ++q)
      if (q == g) r = v[q];
    return r;
  };
  int par = 0;
  int lastpar[G];
  double prev_n[G];
  bool any_block[G];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    lastpar[g] = 0;
    prev_n[g] = 0.0;
    any_block[g] = false;
  }

  // ---- block loop (to the longest chain of the cluster) --------------------
  for (int u0 = 1; u0 <= Lmax; u0 += kLP) {
    int nPq[G];
    double ncq[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const int n = Lq[g] - u0 + 1;
      nPq[g] = n < 0 ? 0 : (n < kLP ? n : kLP);
      ncq[g] = misc0[g * 16 + 1];
    }

    // ===== phase A =====
    if (reinterpret_cast<volatile int*>(anyflag)[0]) {
      for (int i = tid; i < G * RB; i += kNT) {
        const int g = i / RB, cc = i % CL;
        if (cc < Cr && flag0[2 * (g * CL + cc)]) ring0[i] *= 1.0 / fac0[g * CL + cc];
      }
      __syncthreads();
      for (int i = tid; i < G * CL; i += kNT) {
        if (flag0[2 * i]) ref0[i] += log(fac0[i]);
        flag0[2 * i] = 0;
      }
      if (tid == 0) anyflag[0] = 0;
      __syncthreads();
    }
    // inputs of the block's targets
    for (int w = tid; w < G * PB; w += kNT) {
      const int g = w / PB, i = (w % PB) / CL, cc = w % CL;
      if (cc >= Cr || i >= nPq[g]) continue;
      const int u = u0 + i;
      pcu0[w] = cumd(g, u, c0 + cc);
      pto0[w] = toff_at(g, u, c0 + cc);
      pso0[w] = soff_at(g, u, c0 + cc);
    }
    __syncthreads();
    for (int w = tid; w < G * PB; w += kNT) {
      const int g = w / PB, i = (w % PB) / CL, cc = w % CL;
      if (cc >= Cr || i >= nPq[g]) continue;
      const double n_cur = pick_d(ncq, g);
      const double rf = ref0[g * CL + cc];
      const double cu = pcu0[w];
      const double lg_ = pto0[w] + rf + dbmax[cc] + csign * cu - n_cur;
      const double lh_ = colmax[cc] + n_cur + pso0[w] - csign * cu - rf;
      // a clipped factor means the scores span more than the float64 range:
      // flag the launch for the log-domain rerun that follows it
      if (L.ovf && (fabs(lg_) > 700.0 || fabs(lh_) > 700.0)) *L.ovf = 1;
      gf0[w] = exp(fmin(fmax(lg_, -700.0), 700.0));
      hf0[w] = exp(fmin(fmax(lh_, -700.0), 700.0));
    }
    // far sums: sources s in [s_lo, u0-1], kLP accumulators per (chain, label, chunk)
    const int s_hi = u0 - 1;
    const int s_lo = (u0 - kcap) > 0 ? (u0 - kcap) : 0;
    const int ns = s_hi - s_lo + 1;
    const int nsplit = pl.nsplit;
    const int chunk = (ns + nsplit - 1) / nsplit;
    for (int w = tid; w < G * CL * nsplit; w += kNT) {
      const int g = w / (CL * nsplit), rem = w % (CL * nsplit);
      const int cc = rem % CL, j = rem / CL;
      const double* ring_g = ring0 + (size_t)g * RB;
      double acc[kLP];
#pragma unroll
      for (int i = 0; i < kLP; ++i) acc[i] = 0.0;
      const int s_top = s_hi - j * chunk;
      int n = chunk;
      if (s_top - n + 1 < s_lo) n = s_top - s_lo + 1;
      const int nPg = pick_i(nPq, g);
      if (cc < Cr && n > 0 && nPg > 0) {
        double win[kLP];
#pragma unroll
        for (int i = 0; i < kLP; ++i) {
          int k = u0 - s_top + i;
          if (k > pl.kx - 1) k = pl.kx - 1;
          win[i] = dbe_at(k, cc);
        }
        int slot = s_top % R;
        for (int base = 0; base < n; base += kLP) {
#pragma unroll
          for (int r = 0; r < kLP; ++r) {
            const int s = s_top - base - r;
            const double E = (base + r < n) ? ring_g[slot * CL + cc] : 0.0;
#pragma unroll
            for (int i = 0; i < kLP; ++i) acc[i] = fma(E, win[(r + i) % kLP], acc[i]);
            int kn = u0 - s + kLP;
            if (kn > pl.kx - 1) kn = pl.kx - 1;
            win[r % kLP] = dbe_at(kn, cc);
            slot = (slot == 0) ? R - 1 : slot - 1;
          }
        }
      }
      double* pg = part0 + (size_t)g * nsplit * PB;
#pragma unroll
      for (int i = 0; i < kLP; ++i) pg[(j * kLP + i) * CL + cc] = acc[i];
    }
    __syncthreads();
    for (int w = tid; w < G * PB; w += kNT) {
      const int g = w / PB, r = w % PB;
      const double* pg = part0 + (size_t)g * nsplit * PB;
      double s = 0.0;
      for (int j = 0; j < nsplit; ++j) s += pg[j * PB + r];
      far0[w] = s;
    }
    __syncthreads();

    // ===== phase B: the block's targets in order =====
    const int nPme = lt ? pick_i(nPq, gs) : 0;
    const double ncme = lt ? pick_d(ncq, gs) : 0.0;
    int nPmax = 0;
#pragma unroll
    for (int g = 0; g < G; ++g) nPmax = nPmax > nPq[g] ? nPmax : nPq[g];
    double ev[kLP];
#pragma unroll
    for (int i = 0; i < kLP; ++i) ev[i] = 0.0;
    int slot = u0 % R;
#pragma unroll
    for (int i = 0; i < kLP; ++i) {
      if (i < nPmax) {
        const int u = u0 + i;
        const bool on = cv && i < nPme;
        double a = 0.0;
        if (on) {
          const int w = (gs * kLP + i) * CL + c;
          double S = far0[w];
#pragma unroll
          for (int j = 2; j <= i; ++j) S = fma(ev[i - j], dbj[j], S);
          if (i >= 1) S = fma(ev[i - 1], dbj[1], S);
          a = (S > 0.0) ? gf0[w] * S : 0.0;
        }
        publish(a, par, on);
        const double ym = matvec(par);
        if (on) {
          const double e = (ym > 0.0) ? ym * hf0[(gs * kLP + i) * CL + c] : 0.0;
          ev[i] = e;
          if (L.ovf && !(isfinite(a) && isfinite(e))) *L.ovf = 1;
          ring_me[slot * CL + c] = e;
          const int t = cpos(gs, u);
          if (atab_me) atab_me[(size_t)t * C + gcl] = a;
          if (Atab_me) Atab_me[(size_t)t * C + gcl] = ym * ecol;
        }
        if (rank == 0 && lt && c == 0 && i < nPme && A.n_tab)
          A.n_tab[(size_t)bq[gs] * (T + 1) + cpos(gs, u)] = ncme;
#pragma unroll
        for (int g = 0; g < G; ++g)
          if (i < nPq[g]) lastpar[g] = par;
        par ^= 1;
        slot = (slot + 1 == R) ? 0 : slot + 1;
      }
    }
    // re-anchor check on the newest source, and the next block's normalisers
    // from the full state vector of each chain's last target
    if (cv && nPme > 0) {
      double e = ev[0];
#pragma unroll
      for (int i = 1; i < kLP; ++i)
        if (i == nPme - 1) e = ev[i];
      if (e > kHi || (e > 0.0 && e < kLo)) {
        flag0[2 * (gs * CL + c)] = 1;
        fac0[gs * CL + c] = e;
        anyflag[0] = 1;
      }
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
      if (warp == g && nPq[g] > 0) {
        const double m = vec_max(abv(lastpar[g], g));
        if (lane == 0) misc0[g * 16 + 1] = ncq[g] + (m > 0.0 ? log(m) : 0.0);
      }
      if (nPq[g] > 0) {
        prev_n[g] = ncq[g];
        any_block[g] = true;
      }
    }
    __syncthreads();
  }

  // ---- outputs ------------------------------------------------------------
  if (dir == 0 && rank == 0) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      if (warp != g || bq[g] >= L.B) continue;
      // logZ = n(L) + log sum_c a[L,c]; n(L) is the normaliser of L's block
      const double s = any_block[g] ? vec_sum(abv(lastpar[g], g)) : 0.0;
      if (lane == 0) {
        const double nL = any_block[g] ? prev_n[g] : misc0[g * 16 + 0];
        const double lz = (Lq[g] == 0 || !(s > 0.0)) ? (double)kRefNegInf : nL + log(s);
        if (A.partition) A.partition[bq[g]] = (float)lz;
        if (A.logz) A.logz[bq[g]] = lz;
      }
    }
  }
}

// How many clusters of lchain_cl_kernel<G> can be resident at once on the
// current device (its GPC layout decides: a cluster's CTAs share one GPC), or
// 0 when the query fails; cached per device.
template <int G>
int max_active_clusters(size_t smem) {
  constexpr int kMaxDev = 64;
  static int cache[kMaxDev] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return 0;
  if (dev < kMaxDev && cache[dev] > 0) return cache[dev];
  if (cudaFuncSetAttribute(lchain_cl_kernel<G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem) != cudaSuccess)
    return 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kNCL * 64);
  cfg.blockDim = dim3(kNT);
  cfg.dynamicSmemBytes = smem;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, (const void*)lchain_cl_kernel<G>, &cfg) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  if (dev < kMaxDev) cache[dev] = n;
  return n;
}

template <int G>
cudaError_t launch_g(const LChainLaunch& L, int nroles, const CPlan& p, cudaStream_t s) {
  const int ngroups = (L.n1 + G - 1) / G;
  const size_t smem = (size_t)p.total * 8;
  cudaError_t e = cudaFuncSetAttribute(lchain_cl_kernel<G>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  lchain_cl_kernel<G><<<nroles * ngroups * kNCL, kNT, smem, s>>>(L, ngroups);
  return cudaGetLastError();
}

}  // namespace

bool lchain_cl_supported(int C, int K) {
  CPlan p;
  return C > 64 && C <= 256 && K >= 1 && cchoose(p, C, K, 1);
}

// nchains = L.n1 (one role) or 2 * L.n1 (roles a0 and a1, L.n1 chains each)
cudaError_t launch_lchain_cl(const LChainLaunch& L, int nchains, cudaStream_t s) {
  if (nchains <= 0 || L.n1 <= 0) return cudaSuccess;
  const int nroles = nchains > L.n1 ? 2 : 1;
  // 1, 2 or 3 chains per cluster (those whose state fits in shared memory):
  // more chains per cluster cost more per position but need fewer clusters,
  // and a cluster that does not fit in the first wave costs a whole second
  // one.  How many clusters are resident at once depends on the device (33
  // of four CTAs on most B200 parts, fewer on some), so it is queried.
  CPlan p1, p2, p3;
  const bool f1 = cchoose(p1, L.C, L.K, 1), f2 = cchoose(p2, L.C, L.K, 2),
             f3 = cchoose(p3, L.C, L.K, 3);
  if (!f1) return cudaErrorInvalidValue;
  // SEMICRF_CLUSTER_CHAINS=1|2|3 forces the count (tests and measurements)
  if (const char* v = getenv("SEMICRF_CLUSTER_CHAINS")) {
    const int g = atoi(v);
    if (g == 3 && f3) return launch_g<3>(L, nroles, p3, s);
    if (g == 2 && f2) return launch_g<2>(L, nroles, p2, s);
    if (g == 1) return launch_g<1>(L, nroles, p1, s);
  }
  auto groups = [&](int g) { return nroles * ((L.n1 + g - 1) / g); };
  // estimated time: waves x the relative cost of one wave with g chains per
  // cluster (1, 1.4, 2.2: measured per position at C = 256, K = 64 on a
  // B200); a failed query assumes the B200's usual 33 resident clusters
  auto waves = [&](int g, int m) {
    if (m <= 0) m = 33;
    return (groups(g) + m - 1) / m;
  };
  const double t1 = waves(1, max_active_clusters<1>((size_t)p1.total * 8)) * 1.0;
  const double t2 = f2 ? waves(2, max_active_clusters<2>((size_t)p2.total * 8)) * 1.4 : 1e30;
  const double t3 = f3 ? waves(3, max_active_clusters<3>((size_t)p3.total * 8)) * 2.2 : 1e30;
  if (t1 <= t2 && t1 <= t3) return launch_g<1>(L, nroles, p1, s);
  if (t2 <= t3) return launch_g<2>(L, nroles, p2, s);
  return launch_g<3>(L, nroles, p3, s);
}

}  // namespace semicrf
