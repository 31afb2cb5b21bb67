// lchain_cl.cu -- float64 log-semiring chain for large label sets
// (64 < C <= 256), one chain per thread-block cluster of four CTAs.
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
// factors, far sums and g/h factors are in shared memory.  Per
// position each CTA computes a[u,c] for its labels, stores them into all four
// CTAs' shared memory (distributed shared memory), and one cluster barrier
// later every CTA holds the full vector a[u,.] and computes its slice of the
// mat-vec.  The block normaliser and log Z are read off that same vector, so
// they need no further exchange.  The state vector is double-buffered, so the
// one barrier per position also orders its reuse.
//
// Whole chains only (mode 0): no reference ring-checkpoint output and no
// restart records; those run on lchain.cu.  The tables written (a, A, n per
// position) are identical in meaning to lchain.cu's, so lmarg.cu derives the
// gradients unchanged.

#include <cooperative_groups.h>

#include "semicrf_internal.cuh"

namespace semicrf {

namespace {

namespace cg = cooperative_groups;

constexpr int kNT = 512;
constexpr int kNCL = 4;  // CTAs per cluster (chain)
constexpr int kMQ = 32;  // most Mx inputs one thread holds (C <= 256)
constexpr int kLP = 4;   // targets per block
constexpr size_t kSmemMax = 227 * 1024;
constexpr double kHi = 1e78, kLo = 1e-78;  // re-anchor when the newest source leaves this

struct CPlan {
  int C, CL, CPAD, K, kcap, R, kx, nparts, qper, nsplit;
  bool db_smem;
  // offsets in doubles
  int o_ring, o_abuf, o_ypart, o_g, o_h, o_far, o_part, o_pcu, o_pto, o_pso, o_dbe,
      o_dbmax, o_colmax, o_ref, o_fac, o_flag, o_misc, total;
};

__host__ __device__ inline void cmake(CPlan& p, int C, int K, bool db_smem) {
  p.C = C;
  p.CL = (C + kNCL - 1) / kNCL;
  p.K = K;
  p.kcap = K > 1 ? K - 1 : 1;
  p.R = p.kcap + kLP;
  p.kx = p.kcap + kPrepRowsExtra;
  p.nparts = kNT / p.CL;
  p.qper = (C + p.nparts - 1) / p.nparts;
  p.nsplit = kNT / p.CL;
  // state buffer length: the mat-vec reads inputs in groups of four up to
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
  p.o_ring = take(p.R * p.CL);
  p.o_abuf = take(2 * p.CPAD);
  p.o_ypart = take(p.nparts * p.CL);
  p.o_g = take(kLP * p.CL);
  p.o_h = take(kLP * p.CL);
  p.o_far = take(kLP * p.CL);
  p.o_part = take(p.nsplit * kLP * p.CL);
  p.o_pcu = take(kLP * p.CL);
  p.o_pto = take(kLP * p.CL);
  p.o_pso = take(kLP * p.CL);
  p.o_dbe = db_smem ? take(p.kx * p.CL) : -1;
  p.o_dbmax = take(p.CL);
  p.o_colmax = take(p.CL);
  p.o_ref = take(p.CL);
  p.o_fac = take(p.CL);
  p.o_flag = take(p.CL);  // ints, one double each
  p.o_misc = take(16);
  p.total = o;
}

__host__ __device__ inline bool cchoose(CPlan& p, int C, int K) {
  cmake(p, C, K, true);
  if ((size_t)p.total * 8 <= kSmemMax) return true;
  cmake(p, C, K, false);
  return (size_t)p.total * 8 <= kSmemMax;
}

__global__ void __cluster_dims__(kNCL, 1, 1) __launch_bounds__(kNT, 1)
    lchain_cl_kernel(const __grid_constant__ LChainLaunch L) {
  extern __shared__ __align__(16) double csm[];
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int chain = (int)blockIdx.x / kNCL;
  const bool role1 = chain >= L.n1;
  const LChainArgs& A = role1 ? L.a1 : L.a0;
  const int b = role1 ? chain - L.n1 : chain;
  if (b >= L.B) return;  // the same for all CTAs of the cluster
  const int C = L.C, K = L.K, T = L.T;
  const int dir = A.dir;
  const double csign = dir == 0 ? 1.0 : -1.0;
  const long long lraw = A.lengths[b];
  const int Lb = lraw < 0 ? 0 : (lraw > T ? T : (int)lraw);

  CPlan pl;
  cchoose(pl, C, K);
  const int CL = pl.CL, kcap = pl.kcap, R = pl.R;
  const int c0 = rank * CL;
  const int Cr = C - c0 < CL ? (C - c0 > 0 ? C - c0 : 0) : CL;  // labels of this CTA
  double* ring = csm + pl.o_ring;
  double* abuf = csm + pl.o_abuf;
  double* ypart = csm + pl.o_ypart;
  double* gf = csm + pl.o_g;
  double* hf = csm + pl.o_h;
  double* far = csm + pl.o_far;
  double* part = csm + pl.o_part;
  double* pcu = csm + pl.o_pcu;
  double* pto = csm + pl.o_pto;
  double* pso = csm + pl.o_pso;
  double* dbes = pl.db_smem ? csm + pl.o_dbe : nullptr;
  double* dbmax = csm + pl.o_dbmax;
  double* colmax = csm + pl.o_colmax;
  double* ref = csm + pl.o_ref;
  double* fac = csm + pl.o_fac;
  int* flag = reinterpret_cast<int*>(csm + pl.o_flag);
  double* misc = csm + pl.o_misc;
  int* anyflag = reinterpret_cast<int*>(misc + 5);

  const float* cum_b = A.cum + (size_t)b * (T + 1) * C;
  const float* ps_b = A.ps ? A.ps + (size_t)b * T * C : nullptr;
  const float* pe_b = A.pe ? A.pe + (size_t)b * T * C : nullptr;
  auto cpos = [&](int u) { return dir == 0 ? u : Lb - u; };
  // offsets and cum of global label gc at chain position u
  auto soff_at = [&](int u, int gc) -> double {
    const int t = cpos(u);
    if (dir == 0) return (ps_b && t < T) ? (double)ps_b[(size_t)t * C + gc] : 0.0;
    return (pe_b && t >= 1) ? (double)pe_b[(size_t)(t - 1) * C + gc] : 0.0;
  };
  auto toff_at = [&](int u, int gc) -> double {
    const int t = cpos(u);
    if (dir == 0) return (pe_b && t >= 1) ? (double)pe_b[(size_t)(t - 1) * C + gc] : 0.0;
    return (ps_b && t < T) ? (double)ps_b[(size_t)t * C + gc] : 0.0;
  };
  auto cumd = [&](int u, int gc) -> double { return (double)cum_b[(size_t)cpos(u) * C + gc]; };
  auto dbe_at = [&](int k, int i) -> double {
    return pl.db_smem ? dbes[k * CL + i] : L.dbe[(size_t)k * C + c0 + i];
  };

  // ---- constants ----------------------------------------------------------
  if (tid == 0) anyflag[0] = 0;
  for (int i = tid; i < 2 * pl.CPAD; i += kNT) abuf[i] = 0.0;
  for (int i = tid; i < CL; i += kNT) {
    dbmax[i] = i < Cr ? (double)L.dbmax[c0 + i] : 0.0;
    colmax[i] = i < Cr ? (double)A.colmax[c0 + i] : 0.0;
    flag[2 * i] = 0;
  }
  if (pl.db_smem)
    for (int i = tid; i < pl.kx * CL; i += kNT) {
      const int k = i / CL, o = i % CL;
      dbes[i] = o < Cr ? L.dbe[(size_t)k * C + c0 + o] : 0.0;
    }
  __syncthreads();

  const int c = tid;  // serial threads: this CTA's label c (global c0 + c)
  const bool cv = c < Cr;
  const int gcl = c0 + c;
  double dbj[kLP + 1];
#pragma unroll
  for (int j = 0; j <= kLP; ++j) dbj[j] = (cv && j >= 1) ? dbe_at(j, c) : 0.0;
  const double ecol = cv ? exp(colmax[c]) : 0.0;
  double* atab_b = A.a_tab ? A.a_tab + (size_t)b * (T + 1) * C : nullptr;
  double* Atab_b = A.A_tab ? A.A_tab + (size_t)b * (T + 1) * C : nullptr;
  double* ntab_b = A.n_tab ? A.n_tab + (size_t)b * (T + 1) : nullptr;

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
  // ym for this CTA's labels from the full state vector av[0..C): every
  // thread sums its slice of the inputs for one label, then the slices add up
  auto matvec = [&](const double* av) -> double {
    if (mp < pl.nparts) {
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
      ypart[mp * CL + mo] = (y0 + y1) + (y2 + y3);
    }
    __syncthreads();
    double ym = 0.0;
    if (tid < CL)
      for (int p = 0; p < pl.nparts; ++p) ym += ypart[p * CL + tid];
    return ym;
  };
  // store this CTA's a values into buffer par of every CTA of the cluster,
  // then wait until all four CTAs have done so
  auto publish = [&](double a, int par) {
    if (cv) {
#pragma unroll
      for (int r = 0; r < kNCL; ++r) {
        double* dst = cluster.map_shared_rank(abuf + par * pl.CPAD, r);
        dst[gcl] = a;
      }
    }
    cluster.sync();
  };
  // max and sum over the full state vector (read by warp 0)
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
    double a0, ym0;
    if (dir == 0) {
      // alpha[0] = 0 for every label, n = 0: the full vector is known locally
      for (int q = tid; q < C; q += kNT) abuf[q] = 1.0;
      __syncthreads();
      a0 = cv ? 1.0 : 0.0;
      ym0 = matvec(abuf);
    } else {
      a0 = 0.0;
      ym0 = cv ? exp(-colmax[c]) : 0.0;  // beta[Lb] = 0
    }
    if (cv) {
      const double so = soff_at(0, gcl);
      const double cu = cumd(0, gcl);
      ref[c] = (ym0 > 0.0) ? log(ym0) + colmax[c] + so - csign * cu : 0.0;
      ring[0 * CL + c] = (ym0 > 0.0) ? 1.0 : 0.0;
      const int t0 = cpos(0);
      if (atab_b) atab_b[(size_t)t0 * C + gcl] = a0;
      if (Atab_b) Atab_b[(size_t)t0 * C + gcl] = ym0 * ecol;
    }
    if (tid == 0) {
      misc[0] = 0.0;  // n of position 0
      misc[1] = 0.0;  // n of the first block: log max a[0] = 0 (alpha) or 0 (beta)
      if (rank == 0 && ntab_b) ntab_b[cpos(0)] = 0.0;
    }
  }
  // every CTA's constants are in place before any remote store reaches it
  cluster.sync();

  auto prefetch = [&](int u0n) {
    if (u0n > Lb) return;
    const int nPn = (Lb - u0n + 1) < kLP ? (Lb - u0n + 1) : kLP;
    for (int w = tid; w < nPn * CL; w += kNT) {
      const int i = w / CL, cc = w % CL;
      if (cc >= Cr) continue;
      const int u = u0n + i;
      pcu[i * CL + cc] = cumd(u, c0 + cc);
      pto[i * CL + cc] = toff_at(u, c0 + cc);
      pso[i * CL + cc] = soff_at(u, c0 + cc);
    }
  };

  int par = 0, lastpar = 0;
  double prev_n = 0.0;
  bool any_block = false;

  // ---- block loop ---------------------------------------------------------
  for (int u0 = 1; u0 <= Lb; u0 += kLP) {
    const int nP = (Lb - u0 + 1) < kLP ? (Lb - u0 + 1) : kLP;
    const double n_cur = misc[1];

    // ===== phase A =====
    if (reinterpret_cast<volatile int*>(anyflag)[0]) {
      for (int i = tid; i < R * CL; i += kNT) {
        const int cc = i % CL;
        if (cc < Cr && flag[2 * cc]) ring[i] *= 1.0 / fac[cc];
      }
      __syncthreads();
      for (int i = tid; i < CL; i += kNT) {
        if (flag[2 * i]) ref[i] += log(fac[i]);
        flag[2 * i] = 0;
      }
      if (tid == 0) anyflag[0] = 0;
      __syncthreads();
    }
    prefetch(u0);
    __syncthreads();
    for (int w = tid; w < nP * CL; w += kNT) {
      const int i = w / CL, cc = w % CL;
      if (cc >= Cr) continue;
      const double cu = pcu[i * CL + cc];
      const double lg_ = pto[i * CL + cc] + ref[cc] + dbmax[cc] + csign * cu - n_cur;
      const double lh_ = colmax[cc] + n_cur + pso[i * CL + cc] - csign * cu - ref[cc];
      gf[i * CL + cc] = exp(fmin(fmax(lg_, -700.0), 700.0));
      hf[i * CL + cc] = exp(fmin(fmax(lh_, -700.0), 700.0));
    }
    // far sums: sources s in [s_lo, u0-1], kLP accumulators per (label, chunk)
    const int s_hi = u0 - 1;
    const int s_lo = (u0 - kcap) > 0 ? (u0 - kcap) : 0;
    const int ns = s_hi - s_lo + 1;
    const int nsplit = pl.nsplit;
    const int chunk = (ns + nsplit - 1) / nsplit;
    for (int w = tid; w < CL * nsplit; w += kNT) {
      const int cc = w % CL, j = w / CL;
      double acc[kLP];
#pragma unroll
      for (int i = 0; i < kLP; ++i) acc[i] = 0.0;
      const int s_top = s_hi - j * chunk;
      int n = chunk;
      if (s_top - n + 1 < s_lo) n = s_top - s_lo + 1;
      if (cc < Cr && n > 0) {
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
            const double E = (base + r < n) ? ring[slot * CL + cc] : 0.0;
#pragma unroll
            for (int i = 0; i < kLP; ++i) acc[i] = fma(E, win[(r + i) % kLP], acc[i]);
            int kn = u0 - s + kLP;
            if (kn > pl.kx - 1) kn = pl.kx - 1;
            win[r % kLP] = dbe_at(kn, cc);
            slot = (slot == 0) ? R - 1 : slot - 1;
          }
        }
      }
#pragma unroll
      for (int i = 0; i < kLP; ++i) part[(j * kLP + i) * CL + cc] = acc[i];
    }
    __syncthreads();
    for (int w = tid; w < kLP * CL; w += kNT) {
      const int i = w / CL, cc = w % CL;
      double s = 0.0;
      for (int j = 0; j < nsplit; ++j) s += part[(j * kLP + i) * CL + cc];
      far[i * CL + cc] = s;
    }
    __syncthreads();

    // ===== phase B: the block's targets in order =====
    double ev[kLP];
#pragma unroll
    for (int i = 0; i < kLP; ++i) ev[i] = 0.0;
    int slot = u0 % R;
#pragma unroll
    for (int i = 0; i < kLP; ++i) {
      if (i < nP) {
        const int u = u0 + i;
        double a = 0.0;
        if (cv) {
          double S = far[i * CL + c];
#pragma unroll
          for (int j = 2; j <= i; ++j) S = fma(ev[i - j], dbj[j], S);
          if (i >= 1) S = fma(ev[i - 1], dbj[1], S);
          a = (S > 0.0) ? gf[i * CL + c] * S : 0.0;
        }
        publish(a, par);
        const double ym = matvec(abuf + par * pl.CPAD);
        if (cv) {
          const double e = (ym > 0.0) ? ym * hf[i * CL + c] : 0.0;
          ev[i] = e;
          ring[slot * CL + c] = e;
          const int t = cpos(u);
          if (atab_b) atab_b[(size_t)t * C + gcl] = a;
          if (Atab_b) Atab_b[(size_t)t * C + gcl] = ym * ecol;
        }
        if (rank == 0 && tid == 0 && ntab_b) ntab_b[cpos(u)] = n_cur;
        lastpar = par;
        par ^= 1;
        slot = (slot + 1 == R) ? 0 : slot + 1;
      }
    }
    // re-anchor check on the newest source, and the next block's normaliser
    // from the full state vector of the block's last target
    if (cv) {
      double e = ev[0];
#pragma unroll
      for (int i = 1; i < kLP; ++i)
        if (i == nP - 1) e = ev[i];
      if (e > kHi || (e > 0.0 && e < kLo)) {
        flag[2 * c] = 1;
        fac[c] = e;
        anyflag[0] = 1;
      }
    }
    if (warp == 0) {
      const double m = vec_max(abuf + lastpar * pl.CPAD);
      if (lane == 0) misc[1] = n_cur + (m > 0.0 ? log(m) : 0.0);
    }
    __syncthreads();
    prev_n = n_cur;
    any_block = true;
  }

  // ---- outputs ------------------------------------------------------------
  if (dir == 0 && rank == 0 && warp == 0) {
    // logZ = n(Lb) + log sum_c a[Lb,c]; n(Lb) is the normaliser of Lb's block
    const double s = any_block ? vec_sum(abuf + lastpar * pl.CPAD) : 0.0;
    if (lane == 0) {
      const double nL = any_block ? prev_n : misc[0];
      const double lz = (Lb == 0 || !(s > 0.0)) ? (double)kRefNegInf : nL + log(s);
      if (A.partition) A.partition[b] = (float)lz;
      if (A.logz) A.logz[b] = lz;
    }
  }
}

}  // namespace

bool lchain_cl_supported(int C, int K) {
  CPlan p;
  return C > 64 && C <= 256 && K >= 1 && cchoose(p, C, K);
}

cudaError_t launch_lchain_cl(const LChainLaunch& L, int nchains, cudaStream_t s) {
  if (nchains <= 0) return cudaSuccess;
  CPlan p;
  if (!cchoose(p, L.C, L.K)) return cudaErrorInvalidValue;
  const size_t smem = (size_t)p.total * 8;
  cudaError_t e = cudaFuncSetAttribute(lchain_cl_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  lchain_cl_kernel<<<nchains * kNCL, kNT, smem, s>>>(L);
  return cudaGetLastError();
}

}  // namespace semicrf
