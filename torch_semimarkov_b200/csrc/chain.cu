// chain.cu -- the streaming semi-CRF recurrence on one B200 SM.
//
// Reference semantics: streaming/pytorch_reference.py:116-273 (forward) and
// the beta recursion of :276-525 (backward).  The reference evaluates, for
// every position t and duration k, a (C_dst x C_src) edge block
//     edge = cum[t]-cum[t-k] + db[k] (+proj) + tr^T          (:48-113)
// and reduces over (k, c_src).  Because the transition does not depend on k,
// that reduction factorises exactly:
//     A[s,c]   = LSE_c' ( alpha[s,c'] + tr[c',c] )                (C^2 / pos)
//     alpha[t,c] = cum[t,c] + pe[t-1,c]
//                  + LSE_k ( A[t-k,c] + ps[t-k,c] - cum[t-k,c] + db[k,c] )
// ((K-1)*C per position instead of (K-1)*C^2).  The backward chain is the
// same recurrence run from the end of the sequence with tr transposed:
//     beta[t,c'] = LSE_c ( tr[c',c] + G[t,c] )
//     G[t,c]     = ps[t,c] - cum[t,c]
//                  + LSE_k ( cum[t+k,c] + pe[t+k-1,c] + beta[t+k,c] + db[k,c] )
// In chain coordinates u (u = t forward, u = L - t backward) both read
//     x[u]  = toff(u) + LSE_k ( m[u-k] + soff(u-k) + content(u,u-k) + db[k] )
//     m[u]  = LSE_c' ( x[u,c'] + M[c',c] )
// with x = alpha / G and m = A / beta.
//
// One CTA owns one chain.  Targets are processed in blocks of P positions:
//   phase A (all 256 threads): the "far" part of every target's k-sum -- all
//     sources before the block -- for the P targets of the block at once.
//     In the log semiring each source is exponentiated once per block
//     against a per-(block,label) reference and the P targets are then pure
//     FMAs against exp(db) (no exp per (target, source) pair).  A target
//     whose sum would lose precision to underflow is recomputed exactly.
//   phase B (the C "serial" threads, one per label): the P targets one after
//     the other -- near sources inside the block, the merge, and the C x C
//     mat-vec (exp-domain FMAs against exp(M) staged in shared memory).
// Durations are 1..kcap with kcap = max(1, K-1) and db index min(k, K-1)
// (pytorch_reference.py:89-92, :216), so K = 1 is the HMM case.

#include <cstdio>

#include "semicrf_internal.cuh"

namespace semicrf {

constexpr int kThreads = 256;
constexpr size_t kSmemLimit = 227 * 1024;

// ---------------------------------------------------------------------------
// shared-memory plan (identical on host and device)
// ---------------------------------------------------------------------------
struct Plan {
  int C, K, kcap, P, CP, R, kx, nsplit;
  bool mx_smem, db_smem;
  // offsets in 4-byte words
  int o_mx, o_colmax, o_dbl, o_dbe, o_dbmax, o_srcr, o_cumr, o_farl, o_fark, o_tcum, o_toff,
      o_soff, o_anchor, o_ebuf, o_wred, o_pmax, o_pacc, o_pk, o_nr, o_misc;
  int words;
};

__host__ __device__ inline int round_cp(int C) {
  return C <= 32 ? 32 : C <= 64 ? 64 : C <= 128 ? 128 : 256;
}

__host__ __device__ inline void make_plan(Plan& p, int C, int K, int P, int semiring, bool bp,
                                          bool mx_smem, bool db_smem) {
  p.C = C;
  p.K = K;
  p.kcap = K > 1 ? K - 1 : 1;
  p.P = P;
  p.CP = round_cp(C);
  p.R = p.kcap + P;
  p.kx = p.kcap + P + 1;  // rows used here; the prepared arrays have kcap + 17
  p.nsplit = kThreads / C > 0 ? kThreads / C : 1;
  p.mx_smem = mx_smem;
  p.db_smem = db_smem;
  int w = 0;
  auto take = [&](int n) {
    int o = w;
    w += (n + 3) & ~3;  // 16-byte granules
    return o;
  };
  p.o_mx = mx_smem ? take(C * C) : -1;
  p.o_colmax = take(p.CP);
  p.o_dbl = db_smem ? take(p.kx * C) : -1;
  p.o_dbe = (db_smem && semiring == 0) ? take(p.kx * C) : -1;
  p.o_dbmax = take(p.CP);
  p.o_srcr = take(p.R * C);
  p.o_cumr = take(p.R * C);
  p.o_farl = take(P * p.CP);
  p.o_fark = (semiring == 1 && bp) ? take(P * p.CP) : -1;
  p.o_tcum = take(P * p.CP);
  p.o_toff = take(P * p.CP);
  p.o_soff = take(P * p.CP);
  p.o_anchor = take(p.CP);
  p.o_ebuf = take(p.CP);
  p.o_wred = take(16);
  p.o_pmax = take(p.nsplit * C);
  p.o_pacc = take(p.nsplit * P * C);
  p.o_pk = (semiring == 1 && bp) ? take(p.nsplit * P * C) : -1;
  w = (w + 1) & ~1;  // 8-byte alignment for doubles
  p.o_nr = w;
  w += 2 * p.R;
  p.o_misc = w;
  w += 2 * 4;
  p.words = w;
}

static bool choose_plan(Plan& p, int C, int K, int P, int semiring, bool bp) {
  const bool mx_ok = C <= 128;
  make_plan(p, C, K, P, semiring, bp, mx_ok, true);
  if ((size_t)p.words * 4 <= kSmemLimit) return true;
  make_plan(p, C, K, P, semiring, bp, mx_ok, false);
  if ((size_t)p.words * 4 <= kSmemLimit) return true;
  make_plan(p, C, K, P, semiring, bp, false, false);
  return (size_t)p.words * 4 <= kSmemLimit;
}

int chain_block_size(int C) { return 8; }

size_t chain_smem_bytes(int C, int K, int semiring, bool bp) {
  Plan p;
  if (!choose_plan(p, C, K, chain_block_size(C), semiring, bp)) return 0;
  return (size_t)p.words * 4;
}

bool chain_supported(int C, int K, int semiring, bool bp) {
  return C >= 1 && C <= 256 && K >= 1 && chain_smem_bytes(C, K, semiring, bp) > 0;
}

// ---------------------------------------------------------------------------
// prep kernel: per-launch constants (same for every sequence)
// ---------------------------------------------------------------------------
// column maxima (over sources) of tr and tr^T, and duration-bias maxima
// one warp per label c: the lanes stride over the rows, then a warp maximum
__global__ void prep_max_kernel(const float* __restrict__ tr, const float* __restrict__ db, int K,
                                int C, int kcap, int semiring, Prepared pr) {
  const int c = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (c >= C) return;  // warp-uniform
  float mf = kNegInf, mb = kNegInf, md = kNegInf;
  for (int r = lane; r < C; r += 32) {
    mf = fmaxf(mf, tr[r * C + c]);  // M_f[r][c] = tr[r][c]
    mb = fmaxf(mb, tr[c * C + r]);  // M_b[r][c] = tr[c][r]
  }
  for (int k = 1 + lane; k <= kcap; k += 32) md = fmaxf(md, db[(k < K - 1 ? k : K - 1) * C + c]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    mf = fmaxf(mf, __shfl_xor_sync(0xffffffffu, mf, o));
    mb = fmaxf(mb, __shfl_xor_sync(0xffffffffu, mb, o));
    md = fmaxf(md, __shfl_xor_sync(0xffffffffu, md, o));
  }
  if (lane == 0) {
    pr.colmax_f[c] = semiring == 0 ? mf : 0.f;
    pr.colmax_b[c] = semiring == 0 ? mb : 0.f;
    pr.dbmax[c] = md;
  }
}

// the tables, given the maxima
__global__ void prep_kernel(const float* __restrict__ tr, const float* __restrict__ db, int K,
                            int C, int kcap, int kx, int semiring, Prepared pr) {
  const int tid = blockIdx.x * blockDim.x + threadIdx.x;
  const int nth = gridDim.x * blockDim.x;
  for (int i = tid; i < C * C; i += nth) {
    const int r = i / C, c = i % C;
    const float vf = tr[r * C + c], vb = tr[c * C + r];
    if (semiring == 0) {
      // float64: a float32 exp would perturb every weight by ~6e-8, which
      // long sequences turn into visible gradient error
      pr.mxd_f[i] = exp((double)vf - (double)pr.colmax_f[c]);
      pr.mxd_b[i] = exp((double)vb - (double)pr.colmax_b[c]);
    } else {
      pr.mx_f[i] = vf;
      pr.mx_b[i] = vb;
    }
  }
  for (int i = tid; i < kx * C; i += nth) {
    const int k = i / C, c = i % C;
    float v = kNegInf;
    if (k >= 1 && k <= kcap) v = db[(k < K - 1 ? k : K - 1) * C + c];
    pr.dbl[i] = v;
    if (semiring == 0) pr.dbed[i] = (v == kNegInf) ? 0.0 : exp((double)v - (double)pr.dbmax[c]);
  }
}

cudaError_t launch_prep(const float* tr, const float* db, int K, int C, int kcap, int P,
                        int semiring, const Prepared& prep, cudaStream_t s) {
  const int kx = kcap + kPrepRowsExtra;
  (void)P;
  prep_max_kernel<<<(C + 7) / 8, 256, 0, s>>>(tr, db, K, C, kcap, semiring, prep);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  int work = C * C > kx * C ? C * C : kx * C;
  int grid = (work + 255) / 256;
  if (grid > 1024) grid = 1024;
  prep_kernel<<<grid, 256, 0, s>>>(tr, db, K, C, kcap, kx, semiring, prep);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// the chain kernel
// ---------------------------------------------------------------------------
template <int CP, int P, int SEMI, bool BP>
__global__ void __launch_bounds__(kThreads, 1) chain_kernel(const __grid_constant__ ChainLaunch L) {
  extern __shared__ __align__(16) float sm[];
  constexpr int SW = CP / 32;  // serial warps
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const bool serial = tid < CP;

  const bool role1 = (int)blockIdx.x >= L.n1;
  const ChainArgs& A = role1 ? L.a1 : L.a0;
  const int cta = role1 ? (int)blockIdx.x - L.n1 : (int)blockIdx.x;
  const int C = L.C, K = L.K, T = L.T, kcap = L.kcap;
  const int dir = A.dir;
  const float csign = dir == 0 ? 1.f : -1.f;

  int b, seg;
  if (A.mode == 0) {
    b = cta;
    seg = 0;
  } else {
    b = cta / A.nint;
    seg = cta % A.nint;
  }
  if (b >= L.B) return;
  long long lraw = A.lengths[b];
  const int Lb = lraw < 0 ? 0 : (lraw > T ? T : (int)lraw);

  int u_begin = 0, u_end = Lb;
  if (A.mode == 1) {
    u_begin = seg * A.sint;
    if (u_begin > Lb) return;
    const int last = (seg + 1) * A.sint - 1;
    u_end = last < Lb ? last : Lb;
  }

  Plan pl;
  {
    // the host launched with the plan it chose; rebuild it the same way
    const bool mx_ok = C <= 128;
    make_plan(pl, C, K, P, SEMI, BP, mx_ok, true);
    if ((size_t)pl.words * 4 > kSmemLimit) {
      make_plan(pl, C, K, P, SEMI, BP, mx_ok, false);
      if ((size_t)pl.words * 4 > kSmemLimit) make_plan(pl, C, K, P, SEMI, BP, false, false);
    }
  }
  const int R = pl.R;

  float* mx = pl.mx_smem ? sm + pl.o_mx : const_cast<float*>(A.mx);
  float* colmax = sm + pl.o_colmax;
  float* dbl = pl.db_smem ? sm + pl.o_dbl : L.prep.dbl;
  float* dbe = (SEMI == 0) ? (pl.db_smem ? sm + pl.o_dbe : L.prep.dbe) : nullptr;
  float* dbmax = sm + pl.o_dbmax;
  float* srcr = sm + pl.o_srcr;
  float* cumr = sm + pl.o_cumr;
  float* farl = sm + pl.o_farl;
  int* fark = (SEMI == 1 && BP) ? reinterpret_cast<int*>(sm + pl.o_fark) : nullptr;
  float* tcum = sm + pl.o_tcum;
  float* toff = sm + pl.o_toff;
  float* soff = sm + pl.o_soff;
  float* anchor = sm + pl.o_anchor;
  float* ebuf = sm + pl.o_ebuf;
  float* wred = sm + pl.o_wred;
  float* pmax = sm + pl.o_pmax;
  float* pacc = sm + pl.o_pacc;
  int* pk = (SEMI == 1 && BP) ? reinterpret_cast<int*>(sm + pl.o_pk) : nullptr;
  double* nr = reinterpret_cast<double*>(sm + pl.o_nr);
  double* misc = reinterpret_cast<double*>(sm + pl.o_misc);

  const float* cum_b = A.cum + (size_t)b * (T + 1) * C;
  const float* ps_b = A.ps ? A.ps + (size_t)b * T * C : nullptr;
  const float* pe_b = A.pe ? A.pe + (size_t)b * T * C : nullptr;

  auto cpos = [&](int u) { return dir == 0 ? u : Lb - u; };
  auto soff_at = [&](int u, int c) -> float {  // source-side offset of position u
    const int t = cpos(u);
    if (dir == 0) return (ps_b && t < T) ? ps_b[(size_t)t * C + c] : 0.f;
    return (pe_b && t >= 1) ? pe_b[(size_t)(t - 1) * C + c] : 0.f;
  };
  auto toff_at = [&](int u, int c) -> float {  // target-side offset of position u (u >= 1)
    const int t = cpos(u);
    if (dir == 0) return (pe_b && t >= 1) ? pe_b[(size_t)(t - 1) * C + c] : 0.f;
    return (ps_b && t < T) ? ps_b[(size_t)t * C + c] : 0.f;
  };

  // ---- stage per-launch constants -----------------------------------------
  const float* colmax_g = A.colmax;
  for (int i = tid; i < CP; i += kThreads) {
    colmax[i] = i < C ? colmax_g[i] : 0.f;
    dbmax[i] = i < C ? L.prep.dbmax[i] : 0.f;
  }
  if (pl.mx_smem)
    for (int i = tid; i < C * C; i += kThreads) mx[i] = A.mx[i];
  if (pl.db_smem) {
    for (int i = tid; i < pl.kx * C; i += kThreads) dbl[i] = L.prep.dbl[i];
    if (SEMI == 0)
      for (int i = tid; i < pl.kx * C; i += kThreads) dbe[i] = L.prep.dbe[i];
  }
  const bool fwd_full = (dir == 0 && A.mode == 0);
  if (fwd_full && A.ref_ckpt) {
    float* rc = A.ref_ckpt + (size_t)b * A.nref * K * C;
    const int n = A.nref * K * C;
    for (int i = tid; i < n; i += kThreads) rc[i] = (i < C) ? 0.f : kRefNegInf;
  }
  __syncthreads();

  // per-thread constants of the serial label c
  const int c = tid;
  const bool cv = serial && c < C;
  float dblr[P];
#pragma unroll
  for (int j = 0; j < P; ++j) dblr[j] = (cv && j >= 1) ? dbl[j * C + c] : kNegInf;

  float* tabx_b = A.tab_x ? A.tab_x + (size_t)b * (T + 1) * C : nullptr;
  float* tabm_b = A.tab_m ? A.tab_m + (size_t)b * (T + 1) * C : nullptr;
  double* tabn_b = A.tab_n ? A.tab_n + (size_t)b * (T + 1) : nullptr;

  // ---- serial-group helpers -----------------------------------------------
  auto sync_serial = [&]() {
    if (SW == 1)
      __syncwarp();
    else
      named_barrier(1, CP);
  };
  auto group_max = [&](float v) -> float {  // max over the serial group
    float m = warp_max(v);
    if (SW == 1) return m;
    if (lane == 0) wred[warp] = m;
    named_barrier(1, CP);
    float r = wred[0];
#pragma unroll
    for (int w = 1; w < SW; ++w) r = fmaxf(r, wred[w]);
    named_barrier(1, CP);
    return r;
  };
  auto group_sum = [&](float v) -> float {
    float s = warp_sum(v);
    if (SW == 1) return s;
    if (lane == 0) wred[8 + warp] = s;
    named_barrier(1, CP);
    float r = 0.f;
#pragma unroll
    for (int w = 0; w < SW; ++w) r += wred[8 + w];
    named_barrier(1, CP);
    return r;
  };
  // mat-vec: m[c] = LSE_c'( x[c'] + M[c'][c] ) (log) or max with argmax.
  auto matvec = [&](float xv, int& arg) -> float {
    float res;
    arg = 0;
    if (SEMI == 0) {
      const float mxv = group_max(cv ? xv : kNegInf);
      const float e = (cv && mxv != kNegInf) ? ex(xv - mxv) : 0.f;
      ebuf[c] = e;
      sync_serial();
      float y0 = 0.f, y1 = 0.f, y2 = 0.f, y3 = 0.f;
      if (cv) {
        int q = 0;
        for (; q + 4 <= C; q += 4) {
          y0 = fmaf(ebuf[q + 0], mx[(q + 0) * C + c], y0);
          y1 = fmaf(ebuf[q + 1], mx[(q + 1) * C + c], y1);
          y2 = fmaf(ebuf[q + 2], mx[(q + 2) * C + c], y2);
          y3 = fmaf(ebuf[q + 3], mx[(q + 3) * C + c], y3);
        }
        for (; q < C; ++q) y0 = fmaf(ebuf[q], mx[q * C + c], y0);
      }
      const float y = (y0 + y1) + (y2 + y3);
      res = (cv && y > 0.f) ? mxv + colmax[c] + lg(y) : kNegInf;
      sync_serial();
    } else {
      ebuf[c] = cv ? xv : kNegInf;
      sync_serial();
      float best = kNegInf;
      if (cv) {
        for (int q = 0; q < C; ++q) {
          const float v = ebuf[q] + mx[q * C + c];
          if (v > best) {
            best = v;
            arg = q;
          }
        }
      }
      res = best;
      sync_serial();
    }
    return res;
  };

  // ---- initial state ------------------------------------------------------
  float xlast = kNegInf;  // x of the last processed position (serial threads)
  if (A.mode == 0 || seg == 0) {
    // fresh start at u = 0
    if (serial) {
      float xh0, mh0;
      int arg = 0;
      if (dir == 0) {
        xh0 = 0.f;
        mh0 = matvec(0.f, arg);
      } else {
        xh0 = kNegInf;
        mh0 = 0.f;
      }
      if (cv) {
        srcr[0 * C + c] = mh0 + soff_at(0, c);
        cumr[0 * C + c] = cum_b[(size_t)cpos(0) * C + c];
        const int t0 = cpos(0);
        if (tabx_b && dir == 0) tabx_b[(size_t)t0 * C + c] = xh0;
        if (tabm_b) tabm_b[(size_t)t0 * C + c] = mh0;
        if (BP && SEMI == 1 && A.bp_c && dir == 0)
          A.bp_c[((size_t)b * (T + 1) + t0) * C + c] = (uint8_t)arg;
      }
      if (tid == 0) {
        nr[0] = 0.0;
        if (tabn_b) tabn_b[cpos(0)] = 0.0;
      }
      xlast = (dir == 0 && cv) ? 0.f : kNegInf;
    }
  } else {
    // restart from a saved checkpoint at u_begin = seg * sint
    const size_t rec = (size_t)kcap * C + 2 * C;
    const float* svf = A.sv_f + ((size_t)b * A.nint + seg) * rec;
    const double* svd = A.sv_d + ((size_t)b * A.nint + seg) * kcap;
    for (int i = tid; i < kcap * C; i += kThreads) {
      const int j = i / C, cc = i % C;
      const int s = u_begin - j;
      if (s >= 0) {
        srcr[(s % R) * C + cc] = svf[i];
        cumr[(s % R) * C + cc] = cum_b[(size_t)cpos(s) * C + cc];
      }
    }
    for (int j = tid; j < kcap; j += kThreads) {
      const int s = u_begin - j;
      if (s >= 0) nr[s % R] = svd[j];
    }
    __syncthreads();
    if (serial) {
      const float xh0 = cv ? svf[(size_t)kcap * C + c] : kNegInf;
      const float mh0 = cv ? svf[(size_t)kcap * C + C + c] : kNegInf;
      const int t0 = cpos(u_begin);
      if (cv) {
        if (tabx_b) tabx_b[(size_t)t0 * C + c] = xh0;
        if (tabm_b) tabm_b[(size_t)t0 * C + c] = mh0;
      }
      if (tid == 0 && tabn_b) tabn_b[t0] = nr[u_begin % R];
      xlast = xh0;
    }
  }
  // first block normaliser: N(u_begin) + rint(max_c x[u_begin])
  if (serial) {
    const float m = group_max(xlast);
    if (tid == 0) {
      const double nb = (m == kNegInf || !(m == m)) ? 0.0 : (double)rintf(m);
      misc[0] = nr[u_begin % R] + nb;
    }
  }
  __syncthreads();
  double n_cur = misc[0];

  // ---- block loop ---------------------------------------------------------
  for (int u0 = u_begin + 1; u0 <= u_end; u0 += P) {
    const int nP = (u_end - u0 + 1) < P ? (u_end - u0 + 1) : P;

    // ===== phase A: preload target data and far sums (all threads) =====
    for (int i = tid; i < P * CP; i += kThreads) {
      const int ii = i / CP, cc = i % CP;
      if (cc < C && ii < nP) {
        const int u = u0 + ii;
        tcum[ii * CP + cc] = cum_b[(size_t)cpos(u) * C + cc];
        toff[ii * CP + cc] = toff_at(u, cc);
        soff[ii * CP + cc] = soff_at(u, cc);
      }
    }
    for (int i = tid; i < C; i += kThreads) anchor[i] = cum_b[(size_t)cpos(u0) * C + i];
    __syncthreads();

    const int s_hi = u0 - 1;
    const int s_lo = (u0 - kcap) > 0 ? (u0 - kcap) : 0;
    const int ns = s_hi - s_lo + 1;  // >= 1
    const int nsplit = pl.nsplit;
    const int chunk = (ns + nsplit - 1) / nsplit;
    for (int w = tid; w < C * nsplit; w += kThreads) {
      const int cc = w % C, j = w / C;
      const int s_top = s_hi - j * chunk;
      int n = chunk;
      if (s_top - n + 1 < s_lo) n = s_top - s_lo + 1;
      const float anc = anchor[cc];
      if (SEMI == 0) {
        float acc[P];
#pragma unroll
        for (int i = 0; i < P; ++i) acc[i] = 0.f;
        float lmax = kNegInf;
        if (n > 0) {
          float win[P];
#pragma unroll
          for (int i = 0; i < P; ++i) {
            int k = u0 - s_top + i;
            if (k > pl.kx - 1) k = pl.kx - 1;
            win[i] = dbe[k * C + cc];
          }
          for (int base = 0; base < n; base += P) {
#pragma unroll
            for (int r = 0; r < P; ++r) {
              const int s = s_top - base - r;
              float E = 0.f;
              if (base + r < n) {
                const int sl = s % R;
                const float e = ((float)(nr[sl] - n_cur) + (anc - cumr[sl * C + cc]) * csign) +
                                srcr[sl * C + cc];
                if (e != kNegInf) {
                  if (e > lmax) {
                    const float f = (lmax == kNegInf) ? 0.f : ex(lmax - e);
#pragma unroll
                    for (int i = 0; i < P; ++i) acc[i] *= f;
                    lmax = e;
                  }
                  E = ex(e - lmax);
                }
              }
#pragma unroll
              for (int i = 0; i < P; ++i) acc[i] = fmaf(E, win[(r + i) % P], acc[i]);
              int kn = u0 - s + P;
              if (kn > pl.kx - 1) kn = pl.kx - 1;
              win[r % P] = dbe[kn * C + cc];
            }
          }
        }
        pmax[j * C + cc] = lmax;
#pragma unroll
        for (int i = 0; i < P; ++i) pacc[(j * P + i) * C + cc] = acc[i];
      } else {
        float acc[P];
        int kk[P];
#pragma unroll
        for (int i = 0; i < P; ++i) {
          acc[i] = kNegInf;
          kk[i] = 0;
        }
        for (int q = 0; q < n; ++q) {
          const int s = s_top - q;
          const int sl = s % R;
          const float e = ((float)(nr[sl] - n_cur) + (anc - cumr[sl * C + cc]) * csign) +
                          srcr[sl * C + cc];
#pragma unroll
          for (int i = 0; i < P; ++i) {
            const int k = u0 + i - s;
            const float v = e + dbl[(k < pl.kx ? k : pl.kx - 1) * C + cc];
            if (v > acc[i]) {
              acc[i] = v;
              kk[i] = k;
            }
          }
        }
#pragma unroll
        for (int i = 0; i < P; ++i) {
          pacc[(j * P + i) * C + cc] = acc[i];
          if (BP) pk[(j * P + i) * C + cc] = kk[i];
        }
      }
    }
    __syncthreads();

    // reduce the nsplit partials of every (target, label)
    for (int w = tid; w < P * C; w += kThreads) {
      const int ii = w / C, cc = w % C;
      float far;
      int fk = 0;
      if (SEMI == 0) {
        float m = kNegInf;
        for (int j = 0; j < nsplit; ++j) m = fmaxf(m, pmax[j * C + cc]);
        if (m == kNegInf) {
          far = kNegInf;
        } else {
          float ssum = 0.f;
          for (int j = 0; j < nsplit; ++j) {
            const float pm = pmax[j * C + cc];
            if (pm != kNegInf) ssum = fmaf(pacc[(j * P + ii) * C + cc], ex(pm - m), ssum);
          }
          if (ssum >= 8.0e-28f) {  // 2^-90: all that underflowed is < 2^-36 of the sum
            far = m + dbmax[cc] + lg(ssum);
          } else {
            // exact log-domain evaluation of this target's far sum
            const int u = u0 + ii;
            float mm = kNegInf;
            for (int s = s_hi; s >= s_lo; --s) {
              const int k = u - s;
              if (k > kcap) break;
              const int sl = s % R;
              const float v = ((float)(nr[sl] - n_cur) + (anchor[cc] - cumr[sl * C + cc]) * csign) +
                              srcr[sl * C + cc] + dbl[k * C + cc];
              mm = fmaxf(mm, v);
            }
            if (mm == kNegInf) {
              far = kNegInf;
            } else {
              float acc = 0.f;
              for (int s = s_hi; s >= s_lo; --s) {
                const int k = u - s;
                if (k > kcap) break;
                const int sl = s % R;
                const float v =
                    ((float)(nr[sl] - n_cur) + (anchor[cc] - cumr[sl * C + cc]) * csign) +
                    srcr[sl * C + cc] + dbl[k * C + cc];
                acc += ex(v - mm);
              }
              far = mm + lg(acc);
            }
          }
        }
      } else {
        far = kNegInf;
        for (int j = 0; j < nsplit; ++j) {  // chunk 0 holds the newest sources (smallest k)
          const float v = pacc[(j * P + ii) * C + cc];
          if (v > far) {
            far = v;
            if (BP) fk = pk[(j * P + ii) * C + cc];
          }
        }
      }
      farl[ii * CP + cc] = far;
      if (BP && SEMI == 1) fark[ii * CP + cc] = fk;
    }
    __syncthreads();

    // ===== phase B: the P targets in order (serial threads) =====
    if (serial) {
      float srcv[P], tcv[P];
      const float anc = cv ? anchor[c] : 0.f;
#pragma unroll
      for (int i = 0; i < P; ++i) {
        srcv[i] = kNegInf;
        tcv[i] = 0.f;
      }
#pragma unroll
      for (int i = 0; i < P; ++i) {
        if (i < nP) {
          const int u = u0 + i;
          const int t = cpos(u);
          const float tci = cv ? tcum[i * CP + c] : 0.f;
          float xh = kNegInf;
          int bk = 0;
          if (cv) {
            const float far = farl[i * CP + c];
            const float farf = (far == kNegInf) ? kNegInf : far + (tci - anc) * csign;
            if (SEMI == 0) {
              float m = farf;
              float tv[P];
#pragma unroll
              for (int j = 1; j <= i; ++j) {
                tv[j] = (tci - tcv[i - j]) * csign + srcv[i - j] + dblr[j];
                m = fmaxf(m, tv[j]);
              }
              if (m != kNegInf) {
                float sacc = (farf == kNegInf) ? 0.f : ex(farf - m);
#pragma unroll
                for (int j = 1; j <= i; ++j) sacc += ex(tv[j] - m);
                xh = toff[i * CP + c] + (m + lg(sacc));
              }
            } else {
              float best = kNegInf;
#pragma unroll
              for (int j = 1; j <= i; ++j) {
                const float v = (tci - tcv[i - j]) * csign + srcv[i - j] + dblr[j];
                if (v > best) {
                  best = v;
                  bk = j;
                }
              }
              if (farf > best) {
                best = farf;
                if (BP) bk = fark[i * CP + c];
              }
              if (best != kNegInf) xh = toff[i * CP + c] + best;
            }
          }
          // outputs that depend on x
          if (cv) {
            if (tabx_b) tabx_b[(size_t)t * C + c] = xh;
            if (BP && SEMI == 1 && A.bp_k)
              A.bp_k[((size_t)b * (T + 1) + t) * C + c] = (int16_t)bk;
            if (fwd_full && A.ref_ckpt) {
              const int S = A.sref;
              const int ic = (u + S - 1) / S;
              if (ic < A.nref && ic * S <= Lb && ic * S - u < K)
                A.ref_ckpt[(((size_t)b * A.nref + ic) * K + (u % K)) * C + c] =
                    (float)((double)xh + n_cur);
            }
          }
          int arg = 0;
          const float mh = matvec(xh, arg);
          if (cv) {
            const float sv = mh + soff[i * CP + c];
            srcv[i] = sv;
            tcv[i] = tci;
            srcr[(u % R) * C + c] = sv;
            cumr[(u % R) * C + c] = tci;
            if (tabm_b) tabm_b[(size_t)t * C + c] = mh;
            if (BP && SEMI == 1 && A.bp_c && dir == 0)
              A.bp_c[((size_t)b * (T + 1) + t) * C + c] = (uint8_t)arg;
          }
          if (tid == 0) {
            nr[u % R] = n_cur;
            if (tabn_b) tabn_b[t] = n_cur;
          }
          xlast = xh;
          // restart state for the backward recompute
          if (fwd_full && A.write_saved && (u % A.sint) == 0) {
            sync_serial();
            const int ic = u / A.sint;
            if (ic < A.nint) {
              const size_t rec = (size_t)kcap * C + 2 * C;
              float* svf = A.sv_f + ((size_t)b * A.nint + ic) * rec;
              double* svd = A.sv_d + ((size_t)b * A.nint + ic) * kcap;
              for (int q = tid; q < kcap * C; q += CP) {
                const int j = q / C, cc = q % C;
                const int s = u - j;
                svf[q] = s >= 0 ? srcr[(s % R) * C + cc] : kNegInf;
              }
              for (int j = tid; j < kcap; j += CP) {
                const int s = u - j;
                svd[j] = s >= 0 ? nr[s % R] : 0.0;
              }
              if (cv) {
                svf[(size_t)kcap * C + c] = xh;
                svf[(size_t)kcap * C + C + c] = mh;
              }
            }
          }
          sync_serial();
        }
      }
      // next block normaliser from the last target of this block
      const float m = group_max(cv ? xlast : kNegInf);
      if (tid == 0) {
        const double nb = (m == kNegInf || !(m == m)) ? 0.0 : (double)rintf(m);
        misc[1] = n_cur + nb;
      }
    }
    __syncthreads();
    n_cur = misc[1];
    __syncthreads();
  }

  // ---- final: partition / Viterbi score ----------------------------------
  if (fwd_full && serial) {
    // x[Lb] is xlast (Lb >= 1) or x[0] = 0 (Lb == 0, reported as NEG_INF)
    const double n_last = nr[Lb % R];
    if (SEMI == 0) {
      const float m = group_max(cv ? xlast : kNegInf);
      const float e = (cv && m != kNegInf) ? ex(xlast - m) : 0.f;
      const float ssum = group_sum(e);
      if (tid == 0) {
        double lz = (Lb == 0 || m == kNegInf) ? (double)kRefNegInf : n_last + (double)m + (double)lg(ssum);
        if (A.partition) A.partition[b] = (float)lz;
        if (A.logz) A.logz[b] = lz;
      }
    } else {
      const float m = group_max(cv ? xlast : kNegInf);
      // first argmax over labels
      int cand = (cv && xlast == m) ? c : 0x7fffffff;
      for (int o = 16; o > 0; o >>= 1) cand = min(cand, __shfl_xor_sync(0xffffffffu, cand, o));
      if (SW > 1) {
        if (lane == 0) reinterpret_cast<int*>(wred)[warp] = cand;
        named_barrier(1, CP);
        int r = reinterpret_cast<int*>(wred)[0];
        for (int w = 1; w < SW; ++w) r = min(r, reinterpret_cast<int*>(wred)[w]);
        cand = r;
      }
      if (tid == 0) {
        const double sc = (Lb == 0 || m == kNegInf) ? (double)kRefNegInf : n_last + (double)m;
        if (A.partition) A.partition[b] = (float)sc;
        if (A.logz) A.logz[b] = sc;
        if (A.score) A.score[b] = (float)sc;
        if (A.final_c) A.final_c[b] = (cand == 0x7fffffff) ? 0 : cand;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// host launcher
// ---------------------------------------------------------------------------
template <int CP, int SEMI, bool BP>
static cudaError_t launch_cp(const ChainLaunch& L, int grid, size_t smem, cudaStream_t s) {
  constexpr int P = 8;
  auto kern = chain_kernel<CP, P, SEMI, BP>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  if (e != cudaSuccess) return e;
  kern<<<grid, kThreads, smem, s>>>(L);
  return cudaGetLastError();
}

template <int SEMI, bool BP>
static cudaError_t launch_semi(const ChainLaunch& L, int grid, size_t smem, cudaStream_t s) {
  const int cp = round_cp(L.C);
  switch (cp) {
    case 32: return launch_cp<32, SEMI, BP>(L, grid, smem, s);
    case 64: return launch_cp<64, SEMI, BP>(L, grid, smem, s);
    case 128: return launch_cp<128, SEMI, BP>(L, grid, smem, s);
    default: return launch_cp<256, SEMI, BP>(L, grid, smem, s);
  }
}

cudaError_t launch_chain(const ChainLaunch& L, int grid, int semiring, bool backpointers,
                         cudaStream_t s) {
  if (grid <= 0) return cudaSuccess;
  Plan p;
  if (!choose_plan(p, L.C, L.K, 8, semiring, backpointers)) return cudaErrorInvalidValue;
  const size_t smem = (size_t)p.words * 4;
  if (semiring == 0) return launch_semi<0, false>(L, grid, smem, s);
  if (backpointers) return launch_semi<1, true>(L, grid, smem, s);
  return launch_semi<1, false>(L, grid, smem, s);
}

}  // namespace semicrf
