// lchain.cu -- log-semiring streaming semi-CRF chain in float64 linear domain.
//
// Reference semantics: streaming/pytorch_reference.py:116-273 (forward) and
// :276-525 (backward).  The recurrence is factorised exactly as described in
// chain.cu:
//     x[u,c] = toff(u,c) + LSE_k ( m[u-k,c] + soff(u-k,c) + db[k,c]
//                                   + csign*(cum(u,c) - cum(u-k,c)) )
//     m[u,c] = LSE_c' ( x[u,c'] + M[c',c] )
// but evaluated in the linear domain in float64, so that no exp/log is on
// the per-position critical path and rounding does not accumulate along the
// sequence (float32 log-domain chains drift like sqrt(T)*eps, far above the
// 1e-5 gradient contract at T = 1e4):
//     a[u,c]  = exp(x[u,c] - n_B)               state, n_B per block of P
//     E[s,c]  = exp(m[s,c] + soff(s,c) - csign*cum(s,c) - ref[c])
//                                               source window (ring)
//     a[u,c]  = g[u,c] * sum_k E[u-k,c] * Db[k,c]
//     ym[u,c] = sum_c' a[u,c'] * Mx[c',c]       (Mx = exp(M - colmax))
//     E[u,c]  = ym[u,c] * h[u,c]
// with Db = exp(db - dbmax) and the per-(position, label) factors
//     g = exp(toff + ref + dbmax + csign*cum(u) - n_B)
//     h = exp(colmax + n_B + soff - csign*cum(u) - ref)
// computed in float64 ahead of each block.  ref[c] is re-anchored (and the
// window rescaled) when the newest source leaves [e^-180, e^180]; entries
// that underflow are > e^-700 below the newest source of every target's
// window, i.e. negligible.  Constants Mx and Db are float32 (a fixed 6e-8
// perturbation of tr/db, not an accumulating error).
//
// One CTA = one chain.  Per block of P targets:
//   phase A (256 threads): re-anchoring, the g/h factors, and the far sums
//           over all sources before the block (P accumulators per (label,
//           source chunk)).
//   phase B (C serial threads): the P targets in order -- near sources,
//           the state, the float64 mat-vec, the new source.
// The same kernel runs the alpha chain (dir = 0) and the beta chain (dir =
// 1: the recurrence reversed, with tr^T and the projections swapped).  Both
// write their tables (a = exp(x - n), A = exp(m - n) and n per position), from
// which lmarg.cu derives every gradient.  This kernel serves any C <= 256,
// checkpoint segments (mode 1) and the reference ring-checkpoint output; the
// warp-specialised lchain_ws.cu is the fast path for whole chains at C <= 64.

#include "semicrf_internal.cuh"

namespace semicrf {

#ifdef SEMICRF_TIMING
__device__ unsigned long long g_tim[256][8];
#define TIM_DECL unsigned long long tim_[8] = {0, 0, 0, 0, 0, 0, 0, 0}; unsigned long long tck_ = 0;
#define TIM_START() (tck_ = clock64())
#define TIM_ADD(i) (tim_[i] += clock64() - tck_, tck_ = clock64())
#define TIM_FLUSH() \
  if (tid == 0 && blockIdx.x < 256) for (int q_ = 0; q_ < 8; ++q_) g_tim[blockIdx.x][q_] = tim_[q_];
#else
#define TIM_DECL
#define TIM_START()
#define TIM_ADD(i)
#define TIM_FLUSH()
#endif

namespace {

constexpr int kNT = 256;
constexpr int kLP = 8;  // targets per block
constexpr size_t kSmemMax = 227 * 1024;
constexpr double kHi = 1e78, kLo = 1e-78;  // re-anchor when the newest source leaves this

struct LPlan {
  int C, CP, K, kcap, R, kx, nsplit;
  bool db_smem, mx_smem;
  // byte offsets
  int o_ring, o_dbe, o_mx, o_dbmax, o_colmax, o_ref, o_g, o_h, o_far, o_part, o_abuf, o_misc,
      o_flag, o_fac, o_pcu, o_pto, o_pso;
  int bytes;
};

__host__ __device__ inline int lround_cp(int C) {
  return C <= 32 ? 32 : C <= 64 ? 64 : C <= 128 ? 128 : 256;
}

__host__ __device__ inline int lblock(int C) { return lround_cp(C) == 256 ? 4 : kLP; }

__host__ __device__ inline void lmake(LPlan& p, int C, int K, bool db_smem, bool mx_smem) {
  const int kLP = lblock(C);  // targets per block for this label count
  p.C = C;
  p.CP = lround_cp(C);
  p.K = K;
  p.kcap = K > 1 ? K - 1 : 1;
  p.R = p.kcap + kLP;
  p.kx = p.kcap + kPrepRowsExtra;  // = kcap + 2*kLP + 1
  p.nsplit = kNT / C > 0 ? kNT / C : 1;
  p.db_smem = db_smem;
  p.mx_smem = mx_smem;
  int o = 0;
  auto take = [&](int n) {
    int r = o;
    o += (n + 15) & ~15;
    return r;
  };
  p.o_ring = take(8 * p.R * C);
  p.o_dbe = db_smem ? take(8 * p.kx * C) : -1;
  p.o_mx = mx_smem ? take(8 * C * C) : -1;
  p.o_dbmax = take(8 * p.CP);
  p.o_colmax = take(8 * p.CP);
  p.o_ref = take(8 * p.CP);
  p.o_g = take(8 * kLP * p.CP);
  p.o_h = take(8 * kLP * p.CP);
  p.o_far = take(8 * kLP * p.CP);
  p.o_part = take(8 * p.nsplit * kLP * C);
  p.o_abuf = take(8 * p.CP);
  p.o_misc = take(8 * 16);
  p.o_flag = take(4 * p.CP);
  p.o_fac = take(8 * p.CP);
  p.o_pcu = take(8 * kLP * p.CP);  // prefetched cum / toff / soff of the next block
  p.o_pto = take(8 * kLP * p.CP);
  p.o_pso = take(8 * kLP * p.CP);
  p.bytes = o;
}

__host__ __device__ inline bool lchoose(LPlan& p, int C, int K) {
  const bool mx = C <= 128;
  lmake(p, C, K, true, mx);
  if ((size_t)p.bytes <= kSmemMax) return true;
  lmake(p, C, K, false, mx);
  if ((size_t)p.bytes <= kSmemMax) return true;
  lmake(p, C, K, false, false);
  return (size_t)p.bytes <= kSmemMax;
}

}  // namespace

bool lchain_supported(int C, int K) {
  LPlan p;
  return C >= 1 && C <= 256 && K >= 1 && lchoose(p, C, K);
}

__host__ __device__ inline size_t saved_rec(int C, int K) {
  const int kcap = K > 1 ? K - 1 : 1;
  return (size_t)kcap * C + 3 * (size_t)C + 1;
}

size_t lchain_saved_doubles(int C, int K) { return saved_rec(C, K); }

// ---------------------------------------------------------------------------
template <int CP>
__global__ void __launch_bounds__(kNT, 1) lchain_kernel(const __grid_constant__ LChainLaunch L) {
  extern __shared__ __align__(16) unsigned char smraw[];
  constexpr int SW = CP / 32;
  constexpr int LP = (CP == 256) ? 4 : kLP;  // targets per block
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const bool serial = tid < CP;
  const bool role1 = (int)blockIdx.x >= L.n1;
  const LChainArgs& A = role1 ? L.a1 : L.a0;
  const int cta = role1 ? (int)blockIdx.x - L.n1 : (int)blockIdx.x;
  const int C = L.C, K = L.K, T = L.T;
  const int dir = A.dir;
  const double csign = dir == 0 ? 1.0 : -1.0;

  int b, seg;
  if (A.mode == 0) {
    b = cta;
    seg = 0;
  } else {
    b = cta / A.nint;
    seg = cta % A.nint;
  }
  if (b >= L.B) return;
  const long long lraw = A.lengths[b];
  const int Lb = lraw < 0 ? 0 : (lraw > T ? T : (int)lraw);
  int u_begin = 0, u_end = Lb;
  if (A.mode == 1) {
    u_begin = seg * A.sint;
    if (u_begin > Lb) return;
    const int last = (seg + 1) * A.sint - 1;
    u_end = last < Lb ? last : Lb;
  }

  LPlan pl;
  lchoose(pl, C, K);
  const int kcap = pl.kcap, R = pl.R;
  double* ring = reinterpret_cast<double*>(smraw + pl.o_ring);
  const double* dbe = pl.db_smem ? reinterpret_cast<double*>(smraw + pl.o_dbe) : L.dbe;
  const double* mx = pl.mx_smem ? reinterpret_cast<double*>(smraw + pl.o_mx) : A.mx;
  double* dbmax = reinterpret_cast<double*>(smraw + pl.o_dbmax);
  double* colmax = reinterpret_cast<double*>(smraw + pl.o_colmax);
  double* ref = reinterpret_cast<double*>(smraw + pl.o_ref);
  double* gf = reinterpret_cast<double*>(smraw + pl.o_g);
  double* hf = reinterpret_cast<double*>(smraw + pl.o_h);
  double* far = reinterpret_cast<double*>(smraw + pl.o_far);
  double* part = reinterpret_cast<double*>(smraw + pl.o_part);
  double* abuf = reinterpret_cast<double*>(smraw + pl.o_abuf);
  double* misc = reinterpret_cast<double*>(smraw + pl.o_misc);
  int* flag = reinterpret_cast<int*>(smraw + pl.o_flag);
  double* fac = reinterpret_cast<double*>(smraw + pl.o_fac);
  double* pcu = reinterpret_cast<double*>(smraw + pl.o_pcu);
  double* pto = reinterpret_cast<double*>(smraw + pl.o_pto);
  double* pso = reinterpret_cast<double*>(smraw + pl.o_pso);

  const float* cum_b = A.cum + (size_t)b * (T + 1) * C;
  const float* ps_b = A.ps ? A.ps + (size_t)b * T * C : nullptr;
  const float* pe_b = A.pe ? A.pe + (size_t)b * T * C : nullptr;
  auto cpos = [&](int u) { return dir == 0 ? u : Lb - u; };
  auto soff_at = [&](int u, int c) -> double {
    const int t = cpos(u);
    if (dir == 0) return (ps_b && t < T) ? (double)ps_b[(size_t)t * C + c] : 0.0;
    return (pe_b && t >= 1) ? (double)pe_b[(size_t)(t - 1) * C + c] : 0.0;
  };
  auto toff_at = [&](int u, int c) -> double {
    const int t = cpos(u);
    if (dir == 0) return (pe_b && t >= 1) ? (double)pe_b[(size_t)(t - 1) * C + c] : 0.0;
    return (ps_b && t < T) ? (double)ps_b[(size_t)t * C + c] : 0.0;
  };
  auto cumd = [&](int u, int c) -> double { return (double)cum_b[(size_t)cpos(u) * C + c]; };

  // ---- constants ----------------------------------------------------------
  if (tid == 0) reinterpret_cast<int*>(misc + 5)[0] = 0;
  for (int i = tid; i < CP; i += kNT) {
    dbmax[i] = i < C ? (double)L.dbmax[i] : 0.0;
    colmax[i] = i < C ? (double)A.colmax[i] : 0.0;
    flag[i] = 0;
  }
  if (pl.db_smem)
    for (int i = tid; i < pl.kx * C; i += kNT)
      const_cast<double*>(dbe)[i] = L.dbe[i];
  if (pl.mx_smem)
    for (int i = tid; i < C * C; i += kNT) const_cast<double*>(mx)[i] = A.mx[i];
  const bool fwd_full = dir == 0 && A.mode == 0;
  float* const ref_ckpt = A.ref_ckpt;
  const int nref = A.nref, sref = A.sref, sint = A.sint, nint = A.nint;
  const bool write_saved = fwd_full && A.write_saved;
  double* const svbase = A.sv;
  if (fwd_full && ref_ckpt) {
    float* rc = ref_ckpt + (size_t)b * nref * K * C;
    for (int i = tid; i < nref * K * C; i += kNT) rc[i] = (i < C) ? 0.f : kRefNegInf;
  }
  __syncthreads();

  // per-thread (serial label c) constants
  const int c = tid;
  const bool cv = serial && c < C;
  double dbj[LP + 1];
#pragma unroll
  for (int j = 0; j <= LP; ++j) dbj[j] = (cv && j >= 1) ? dbe[j * C + c] : 0.0;

  double* atab_b = A.a_tab ? A.a_tab + (size_t)b * (T + 1) * C : nullptr;
  double* Atab_b = A.A_tab ? A.A_tab + (size_t)b * (T + 1) * C : nullptr;
  double* ntab_b = A.n_tab ? A.n_tab + (size_t)b * (T + 1) : nullptr;

  auto sync_serial = [&]() {
    if (SW == 1)
      __syncwarp();
    else
      named_barrier(1, CP);
  };
  // max over the serial group of a non-negative double
  auto group_maxd = [&](double v) -> double {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmax(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (SW == 1) return v;
    if (lane == 0) misc[8 + warp] = v;
    named_barrier(1, CP);
    double r = 0.0;
#pragma unroll
    for (int w = 0; w < SW; ++w) r = fmax(r, misc[8 + w]);
    named_barrier(1, CP);
    return r;
  };
  auto group_sumd = [&](double v) -> double {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (SW == 1) return v;
    if (lane == 0) misc[8 + warp] = v;
    named_barrier(1, CP);
    double r = 0.0;
#pragma unroll
    for (int w = 0; w < SW; ++w) r += misc[8 + w];
    named_barrier(1, CP);
    return r;
  };
  // ym[c] = sum_c' a[c'] Mx[c',c].  For C <= 32 the column of lane c lives in
  // registers (zero-padded to 32) and the sum is fully unrolled.
  constexpr int MXR = (CP == 32) ? 32 : 1;
  double mxr[MXR];
#pragma unroll
  for (int q = 0; q < MXR; ++q) mxr[q] = (CP == 32 && cv && q < C) ? mx[q * C + c] : 0.0;
  const double ecol = cv ? exp(colmax[c]) : 0.0;
  auto matvec = [&](double a) -> double {
    abuf[c] = cv ? a : 0.0;
    sync_serial();
    double y[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) y[q] = 0.0;
    if (CP == 32) {
      const double2* ab2 = reinterpret_cast<const double2*>(abuf);
#pragma unroll
      for (int q = 0; q < 16; ++q) {
        const double2 v = ab2[q];
        y[(2 * q) & 7] = fma(v.x, mxr[2 * q], y[(2 * q) & 7]);
        y[(2 * q + 1) & 7] = fma(v.y, mxr[2 * q + 1], y[(2 * q + 1) & 7]);
      }
    } else if (cv) {
      int q = 0;
      for (; q + 4 <= C; q += 4) {
        y[0] = fma(abuf[q + 0], mx[(q + 0) * C + c], y[0]);
        y[1] = fma(abuf[q + 1], mx[(q + 1) * C + c], y[1]);
        y[2] = fma(abuf[q + 2], mx[(q + 2) * C + c], y[2]);
        y[3] = fma(abuf[q + 3], mx[(q + 3) * C + c], y[3]);
      }
      for (; q < C; ++q) y[0] = fma(abuf[q], mx[q * C + c], y[0]);
    }
    sync_serial();
    return ((y[0] + y[1]) + (y[2] + y[3])) + ((y[4] + y[5]) + (y[6] + y[7]));
  };

  // ---- initial state ------------------------------------------------------
  double a_last = 0.0;  // state of the last processed position (serial threads)
  if (A.mode == 0 || seg == 0) {
    if (serial) {
      double a0, ym0;
      if (dir == 0) {
        a0 = cv ? 1.0 : 0.0;  // alpha[0] = 0, n = 0
        ym0 = matvec(a0);
      } else {
        a0 = 0.0;
        ym0 = cv ? exp(-colmax[c]) : 0.0;  // beta[Lb] = 0
      }
      // anchor: E[0,c] = 1  =>  ref = log(ym0) + colmax + soff - csign*cum(0)
      if (cv) {
        const double so = soff_at(0, c);
        const double cu = cumd(0, c);
        ref[c] = (ym0 > 0.0) ? log(ym0) + colmax[c] + so - csign * cu : 0.0;
        ring[0 * C + c] = (ym0 > 0.0) ? 1.0 : 0.0;
        const int t0 = cpos(0);
        if (atab_b) atab_b[(size_t)t0 * C + c] = a0;
        if (Atab_b) Atab_b[(size_t)t0 * C + c] = ym0 * ecol;
      }
      if (tid == 0) {
        misc[0] = 0.0;  // n of position u_begin
        if (ntab_b) ntab_b[cpos(0)] = 0.0;
      }
      a_last = (dir == 0) ? a0 : 0.0;
    }
  } else {
    // restart from the saved state at u_begin = seg * sint
    const size_t rec = saved_rec(C, K);
    const double* sv = A.sv + ((size_t)b * A.nint + seg) * rec;
    for (int i = tid; i < kcap * C; i += kNT) {
      const int j = i / C, cc = i % C;
      const int s = u_begin - j;
      if (s >= 0) ring[(s % R) * C + cc] = sv[i];
    }
    if (serial && cv) {
      ref[c] = sv[(size_t)kcap * C + c];
      a_last = sv[(size_t)kcap * C + C + c];
      const double y0 = sv[(size_t)kcap * C + 2 * C + c];
      const int t0 = cpos(u_begin);
      if (atab_b) atab_b[(size_t)t0 * C + c] = a_last;
      if (Atab_b) Atab_b[(size_t)t0 * C + c] = y0 * ecol;
    }
    if (tid == 0) {
      misc[0] = sv[(size_t)kcap * C + 3 * C];
      if (ntab_b) ntab_b[cpos(u_begin)] = misc[0];
    }
  }
  __syncthreads();
  // first block normaliser; re-anchor check of the newest source (as the
  // original run did at the end of the block that ended at u_begin)
  if (serial) {
    const double m = group_maxd(cv ? a_last : 0.0);
    if (tid == 0) misc[1] = misc[0] + (m > 0.0 ? log(m) : 0.0);
    if (cv) {
      const double e = ring[(u_begin % R) * C + c];
      if (e > kHi || (e > 0.0 && e < kLo)) {
        flag[c] = 1;
        fac[c] = e;
        reinterpret_cast<int*>(misc + 5)[0] = 1;
      }
    }
  }
  __syncthreads();

  auto prefetch = [&](int u0n, int tlo, int tstep) {
    if (u0n > u_end) return;
    const int nPn = (u_end - u0n + 1) < LP ? (u_end - u0n + 1) : LP;
    for (int w = tlo; w < nPn * C; w += tstep) {
      const int i = w / C, cc = w % C;
      const int u = u0n + i;
      pcu[i * CP + cc] = cumd(u, cc);
      pto[i * CP + cc] = toff_at(u, cc);
      pso[i * CP + cc] = soff_at(u, cc);
    }
  };
  prefetch(u_begin + 1, tid, kNT);
  __syncthreads();

  int prev_u0 = -1, prev_nP = 0;
  double prev_n = 0.0;
  TIM_DECL
  TIM_START();

  // ---- block loop ---------------------------------------------------------
  for (int u0 = u_begin + 1; u0 <= u_end; u0 += LP) {
    const int nP = (u_end - u0 + 1) < LP ? (u_end - u0 + 1) : LP;
    const double n_cur = misc[1];

    // ===== phase A =====
    TIM_ADD(0);
    // re-anchor labels whose newest source drifted out of range (fac = that source)
    if (reinterpret_cast<volatile int*>(misc + 5)[0]) {
      for (int i = tid; i < R * C; i += kNT) {
        const int cc = i % C;
        if (flag[cc]) ring[i] *= 1.0 / fac[cc];
      }
      __syncthreads();
      for (int i = tid; i < C; i += kNT) {
        if (flag[i]) ref[i] += log(fac[i]);
        flag[i] = 0;
      }
      if (tid == 0) reinterpret_cast<int*>(misc + 5)[0] = 0;
      __syncthreads();
    }
    if (CP == kNT) {  // no idle warps to prefetch during phase B
      prefetch(u0, tid, kNT);
      __syncthreads();
    }
    // g / h factors of the block's targets (cum / offsets prefetched into smem)
    for (int w = tid; w < nP * C; w += kNT) {
      const int i = w / C, cc = w % C;
      const double cu = pcu[i * CP + cc];
      const double lg_ = pto[i * CP + cc] + ref[cc] + dbmax[cc] + csign * cu - n_cur;
      const double lh_ = colmax[cc] + n_cur + pso[i * CP + cc] - csign * cu - ref[cc];
      // a clipped factor means the scores span more than the float64 range:
      // flag the launch for the log-domain rerun that follows it
      if (L.ovf && (fabs(lg_) > 700.0 || fabs(lh_) > 700.0)) *L.ovf = 1;
      gf[i * CP + cc] = exp(fmin(fmax(lg_, -700.0), 700.0));
      hf[i * CP + cc] = exp(fmin(fmax(lh_, -700.0), 700.0));
    }
    // far sums: sources s in [s_lo, u0-1], P accumulators per (label, chunk)
    const int s_hi = u0 - 1;
    const int s_lo = (u0 - kcap) > 0 ? (u0 - kcap) : 0;
    const int ns = s_hi - s_lo + 1;
    const int nsplit = pl.nsplit;
    const int chunk = (ns + nsplit - 1) / nsplit;
    for (int w = tid; w < C * nsplit; w += kNT) {
      const int cc = w % C, j = w / C;
      const int s_top = s_hi - j * chunk;
      int n = chunk;
      if (s_top - n + 1 < s_lo) n = s_top - s_lo + 1;
      double acc[LP];
#pragma unroll
      for (int i = 0; i < LP; ++i) acc[i] = 0.0;
      if (n > 0) {
        double win[LP];
#pragma unroll
        for (int i = 0; i < LP; ++i) {
          int k = u0 - s_top + i;
          if (k > pl.kx - 1) k = pl.kx - 1;
          win[i] = dbe[k * C + cc];
        }
        int slot = s_top % R;
        for (int base = 0; base < n; base += LP) {
#pragma unroll
          for (int r = 0; r < LP; ++r) {
            const int s = s_top - base - r;
            const double E = (base + r < n) ? ring[slot * C + cc] : 0.0;
#pragma unroll
            for (int i = 0; i < LP; ++i) acc[i] = fma(E, win[(r + i) % LP], acc[i]);
            int kn = u0 - s + LP;
            if (kn > pl.kx - 1) kn = pl.kx - 1;
            win[r % LP] = dbe[kn * C + cc];
            slot = (slot == 0) ? R - 1 : slot - 1;
          }
        }
      }
#pragma unroll
      for (int i = 0; i < LP; ++i) part[(j * LP + i) * C + cc] = acc[i];
    }
    __syncthreads();
    TIM_ADD(1);
    for (int w = tid; w < LP * C; w += kNT) {
      const int i = w / C, cc = w % C;
      double s = 0.0;
      for (int j = 0; j < nsplit; ++j) s += part[(j * LP + i) * C + cc];
      far[i * CP + cc] = s;
    }
    __syncthreads();

    TIM_ADD(2);
    // ===== phase B =====  (idle warps prefetch the next block meanwhile)
    if (CP < kNT && !serial) prefetch(u0 + LP, tid - CP, kNT - CP);
    if (serial) {
      double ev[LP];
#pragma unroll
      for (int i = 0; i < LP; ++i) ev[i] = 0.0;
      int slot = u0 % R;
#pragma unroll
      for (int i = 0; i < LP; ++i) {
        if (i < nP) {
          const int u = u0 + i;
          double S = 0.0, a = 0.0;
          if (cv) {
            S = far[i * CP + c];
#pragma unroll
            for (int j = 2; j <= i; ++j) S = fma(ev[i - j], dbj[j], S);
            if (i >= 1) S = fma(ev[i - 1], dbj[1], S);
            a = (S > 0.0) ? gf[i * CP + c] * S : 0.0;
          }
          TIM_ADD(3);
          const double ym = matvec(a);
          TIM_ADD(4);
          if (cv) {
            const double e = (ym > 0.0) ? ym * hf[i * CP + c] : 0.0;
            ev[i] = e;
            if (L.ovf && !(isfinite(a) && isfinite(e))) *L.ovf = 1;
            ring[slot * C + c] = e;
            const int t = cpos(u);
            if (atab_b) atab_b[(size_t)t * C + c] = a;
            if (Atab_b) Atab_b[(size_t)t * C + c] = ym * ecol;
            if (fwd_full && ref_ckpt) {
              const int Sr = sref;
              const int ic = (u + Sr - 1) / Sr;
              if (ic < nref && ic * Sr <= Lb && ic * Sr - u < K)
                ref_ckpt[(((size_t)b * nref + ic) * K + (u % K)) * C + c] =
                    (a > 0.0) ? (float)(n_cur + log(a)) : kRefNegInf;
            }
          }
          if (tid == 0 && ntab_b) ntab_b[cpos(u)] = n_cur;
          a_last = a;
          if (write_saved && (u % sint) == 0) {
            sync_serial();
            const int ic = u / sint;
            if (ic < nint) {
              const size_t rec = saved_rec(C, K);
              double* sv = svbase + ((size_t)b * nint + ic) * rec;
              for (int q = tid; q < kcap * C; q += CP) {
                const int j = q / C, cc = q % C;
                const int s = u - j;
                sv[q] = s >= 0 ? ring[(s % R) * C + cc] : 0.0;
              }
              if (cv) {
                sv[(size_t)kcap * C + c] = ref[c];
                sv[(size_t)kcap * C + C + c] = a;
                sv[(size_t)kcap * C + 2 * C + c] = ym;
              }
              if (tid == 0) sv[(size_t)kcap * C + 3 * C] = n_cur;
            }
          }
          slot = (slot + 1 == R) ? 0 : slot + 1;
          TIM_ADD(5);
        }
      }
      // re-anchor check on the newest source, and the next block's normaliser
      if (cv) {
        double e = ev[0];
#pragma unroll
        for (int i = 1; i < LP; ++i)
          if (i == nP - 1) e = ev[i];
        if (e > kHi || (e > 0.0 && e < kLo)) {
          flag[c] = 1;
          fac[c] = e;
          reinterpret_cast<int*>(misc + 5)[0] = 1;
        }
      }
      const double m = group_maxd(cv ? a_last : 0.0);
      if (tid == 0) misc[1] = n_cur + (m > 0.0 ? log(m) : 0.0);
    }
    __syncthreads();
    TIM_ADD(6);
    prev_u0 = u0;
    prev_nP = nP;
    prev_n = n_cur;
  }
  TIM_FLUSH();

  // ---- outputs ------------------------------------------------------------
  if (fwd_full) {
    // logZ = n(Lb) + log sum_c a[Lb,c]; n(Lb) is the normaliser of Lb's block
    __syncthreads();
    if (serial) {
      const double s = group_sumd(cv ? a_last : 0.0);
      if (tid == 0) {
        const double nL = (prev_u0 >= 0) ? prev_n : misc[0];
        const double lz = (Lb == 0 || !(s > 0.0)) ? (double)kRefNegInf : nL + log(s);
        if (A.partition) A.partition[b] = (float)lz;
        if (A.logz) A.logz[b] = lz;
      }
    }
  }
}

// ---------------------------------------------------------------------------
template <int CP>
static cudaError_t launch_cp(const LChainLaunch& L, int grid, size_t smem, cudaStream_t s) {
  auto kern = lchain_kernel<CP>;
  cudaError_t e =
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  kern<<<grid, kNT, smem, s>>>(L);
  return cudaGetLastError();
}

#ifdef SEMICRF_TIMING
extern "C" int semicrf_debug_timing(unsigned long long* out) {
  return (int)cudaMemcpyFromSymbol(out, g_tim, sizeof(g_tim));
}
#endif

cudaError_t launch_lchain(const LChainLaunch& L, int grid, cudaStream_t s) {
  if (grid <= 0) return cudaSuccess;
  LPlan p;
  if (!lchoose(p, L.C, L.K)) return cudaErrorInvalidValue;
  const size_t smem = (size_t)p.bytes;
  switch (lround_cp(L.C)) {
    case 32: return launch_cp<32>(L, grid, smem, s);
    case 64: return launch_cp<64>(L, grid, smem, s);
    case 128: return launch_cp<128>(L, grid, smem, s);
    default: return launch_cp<256>(L, grid, smem, s);
  }
}


}  // namespace semicrf
