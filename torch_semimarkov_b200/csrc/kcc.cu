// kcc.cu -- duration-dependent transitions, transition of shape (K, C, C).
//
// compute_edge_block_streaming indexes transition[k] for a segment of
// duration k (streaming/pytorch_reference.py:104-109), so the previous label's
// weight depends on the new segment's duration and the label mixing cannot be
// taken out of the duration sum.  Each chain position combines every source in
// its window with that duration's own C x C matrix, the reference's O(K C^2)
// per position:
//   alpha[t,c] = cum[t,c] + pe[t-1,c] + (+)_k ( (+)_{c'} (alpha[t-k,c'] + tr[k][c',c])
//                                              + ps[t-k,c] - cum[t-k,c] + db[k,c] )
//   beta[t,c]  = (+)_{k,c2} ( tr[k][c,c2] + ps[t,c2] - cum[t,c2] + db[k,c2]
//                             + cum[t+k,c2] + pe[t+k-1,c2] + beta[t+k,c2] ),   beta[len] = 0
// with (+) = logsumexp (log semiring) or max, alpha[0] = 0 and durations
// k = 1 .. min(K-1, window) (pytorch_reference.py:213, :437-446).  The log
// semiring evaluates each label sum in float64 linear form,
//   (+)_{c'} = n + tf[k][c] + log sum_{c'} exp(alpha[s,c'] - n) exp(tr[k][c',c] - tf[k][c]),
// one dot product and one log per (duration, label) item.  Gradients are the
// segment marginals
//   P(s -> s+k, c' -> c) = exp(alpha[s,c'] + tr[k][c',c] + seg(s,k,c) + beta[s+k,c] - logZ)
// for both semirings, as the reference computes them (pytorch_reference.py:458-499).
//
// Kernels: a chain kernel (one CTA per sequence and direction, (duration,
// label) items spread over the CTA, an online log-sum per thread), the start
// and end marginals per position (grad_cum, grad_proj_*), and a register-tiled
// accumulation of the transition marginals sum_s alpha_lin[s,c'] q[s,k,c]
// followed by a fixed-order reduce (grad_transition, grad_duration_bias).

#include "semicrf_internal.cuh"

namespace semicrf {

namespace {

constexpr int kKT = 256;  // threads per CTA
constexpr int kKC = 32;   // durations per source chunk of the beta chain
constexpr int kJ = 4;     // positions per thread in the start-marginal kernel
constexpr int kTR = 32;   // rows (source labels) per transition tile
constexpr int kTC = 256;  // columns (duration, label) per transition tile
constexpr size_t kSmemMax = 200 * 1024;

__device__ __forceinline__ int seq_len(const int64_t* lengths, int b, int T) {
  const long long l = lengths[b];
  return l < 0 ? 0 : (l > T ? T : (int)l);
}

__device__ __forceinline__ void cp_async8(double* dst, const double* src) {
  const unsigned d = (unsigned)__cvta_generic_to_shared(dst);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" ::"r"(d), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;\n" ::: "memory");
}
__device__ __forceinline__ void cp_async_wait1() {
  asm volatile("cp.async.wait_group 1;\n" ::: "memory");
}

__global__ void kcc_prep_kernel(const float* __restrict__ tr, const float* __restrict__ db, int K,
                                int C, KccPrep pr) {
  const int n = K * C;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const int k = i / C, c = i % C;
    const float* m = tr + (size_t)k * C * C;
    double mf = -INFINITY, mb = -INFINITY;
    for (int q = 0; q < C; ++q) {
      mf = fmax(mf, (double)m[q * C + c]);
      mb = fmax(mb, (double)m[c * C + q]);
    }
    pr.tf[i] = mf;
    pr.tb[i] = mb;
    pr.tdf[i] = mf + (double)db[i];
    for (int q = 0; q < C; ++q) {
      const size_t j = ((size_t)k * C + q) * C + c;
      pr.ef[j] = exp((double)m[q * C + c] - mf);
      pr.eb[j] = exp((double)m[c * C + q] - mb);
      if (pr.rf) {  // max semiring: the weights with the duration bias of the new segment
        pr.rf[j] = (double)m[q * C + c] + (double)db[(size_t)k * C + c];
        pr.rb[j] = (double)m[c * C + q] + (double)db[(size_t)k * C + q];
      }
    }
  }
}

// Shared memory of the chain kernel (offsets in doubles).  The per-duration
// C x C factors E[k] are resident when all K of them fit; otherwise they are
// streamed from L2 in chunks of kc durations through two cp.async buffers, or,
// when not even two single-duration buffers fit (C > ~110), read from L2.  The
// (K, C) tables (tf or tb, and db) are kept as float32, which holds them
// exactly (they are float32 inputs or maxima of them).  The forward chain also
// keeps each source position's start term rn + ps - cum (rso) when room is left.
struct ChainPlan {
  int kc, resident, direct, rso;
  size_t ring, rn, t1, dbs, xs, xm, dt, ct, vals, redm, reds, eb, rso_o, total;
};
__host__ __device__ inline ChainPlan chain_plan(int C, int K) {
  ChainPlan p{};
  const size_t cc = (size_t)C * C, kcs = (size_t)K * C;
  const int kcap = K - 1;
  const int kc_max = kKC < kcap ? kKC : kcap;
  size_t o = 0;
  p.ring = o;
  o += kcs;
  p.rn = o;
  o += K;
  p.t1 = o;
  o += (kcs + 1) / 2;
  p.dbs = o;
  o += (kcs + 1) / 2;
  p.xs = o;
  o += (size_t)kKC * C;
  p.xm = o;
  o += kKC;
  p.dt = o;
  o += C;
  p.ct = o;
  o += C;
  p.vals = o;
  o += C;
  p.redm = o;
  o += kKT;
  p.reds = o;
  o += kKT;
  p.eb = o;
  const size_t cap = kSmemMax / 8;
  if (o + (size_t)K * cc <= cap) {
    p.resident = 1;
    p.kc = kc_max;
    o += (size_t)K * cc;
  } else {
    const size_t with_rso = cap > o + kcs ? (cap - o - kcs) / (2 * cc) : 0;
    const size_t without = cap > o ? (cap - o) / (2 * cc) : 0;
    const size_t want = kc_max < 8 ? kc_max : 8;
    size_t kc = with_rso >= want ? with_rso : without;
    if (kc > (size_t)kc_max) kc = kc_max;
    if (kc >= 1) {
      p.kc = (int)kc;
      o += 2 * kc * cc;
    } else {
      p.direct = 1;
      p.kc = kc_max;
    }
  }
  if (o + kcs <= cap) {
    p.rso = 1;
    p.rso_o = o;
    o += kcs;
  }
  p.total = o;
  return p;
}

// One CTA per (sequence, direction).  Writes log alpha and its row maxima
// (dir 0) or log beta (dir 1) for positions 0 .. len when the tables are given.
// Thread (label c, slot j) = (tid % C, tid / C) handles the durations j, j + G,
// ... of label c (G = 256 / C slots), so the lanes of a warp read one source
// row and adjacent columns of E[k] (no bank conflicts); a position's G
// partial sums per label are combined by one warp per label with shuffles.
template <int SEMI>
__global__ void __launch_bounds__(kKT) kcc_chain_kernel(const KccArgs a) {
  if (a.gate && *a.gate == 0) return;  // fallback pass of the blocked chain, not needed
  extern __shared__ __align__(16) double ksm[];
  const int C = a.C, K = a.K, T = a.T, kcap = a.kcap, R = K;
  const int b = blockIdx.x, dir = blockIdx.y, tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5;
  const int Lb = seq_len(a.lengths, b, T);
  const ChainPlan sp = chain_plan(C, K);
  const size_t cc = (size_t)C * C;
  double* ring = ksm + sp.ring;  // dir 0: alpha rows (linear for log); dir 1: log source rows
  double* rn = ksm + sp.rn;      // dir 0: row maxima of alpha
  float* t1f = reinterpret_cast<float*>(ksm + sp.t1);   // dir 0: tf, dir 1: tb
  float* dbf = reinterpret_cast<float*>(ksm + sp.dbs);  // duration bias
  double* xs = ksm + sp.xs;      // dir 1: one chunk of duration source rows
  double* xm = ksm + sp.xm;
  double* dt = ksm + sp.dt;
  double* ct = ksm + sp.ct;  // cum[t] + pe[t-1] of the position being computed
  double* vals = ksm + sp.vals;
  double* redm = ksm + sp.redm;
  double* reds = ksm + sp.reds;
  double* ebuf = ksm + sp.eb;
  double* rso = ksm + sp.rso_o;  // dir 0 with sp.rso: start term of each ring position
  const bool use_rso = sp.rso && dir == 0;
  __shared__ double s_m;
  const float* cum_b = a.cum + (size_t)b * (T + 1) * C;
  const float* ps_b = a.ps ? a.ps + (size_t)b * T * C : nullptr;
  const float* pe_b = a.pe ? a.pe + (size_t)b * T * C : nullptr;
  auto cu = [&](int t, int c) { return (double)cum_b[(size_t)t * C + c]; };
  auto psv = [&](int t, int c) {
    return (ps_b && t < T) ? (double)ps_b[(size_t)t * C + c] : 0.0;
  };
  auto pev = [&](int t, int c) {
    return (pe_b && t >= 1) ? (double)pe_b[(size_t)(t - 1) * C + c] : 0.0;
  };
  // E[k][q][c]: log semiring exp(tr - max) factors, max semiring raw tr, in the
  // orientation of this direction
  const double* Eg = SEMI == 0 ? (dir == 0 ? a.pr.ef : a.pr.eb) : (dir == 0 ? a.pr.rf : a.pr.rb);
  const bool resident = sp.resident != 0 || sp.direct != 0;  // no staging either way
  const double* Eall = sp.direct ? Eg : ebuf;
  if (sp.resident)
    for (size_t i = tid; i < (size_t)K * cc; i += kKT) ebuf[i] = Eg[i];
  {
    const double* t1g = dir == 0 ? a.pr.tf : a.pr.tb;
    for (int i = tid; i < K * C; i += kKT) {
      t1f[i] = (float)t1g[i];
      dbf[i] = a.db[i];
    }
  }
  if (dir == 0 && a.ref_ckpt) {
    float* rc = a.ref_ckpt + (size_t)b * a.nref * K * C;
    for (size_t i = tid; i < (size_t)a.nref * K * C; i += kKT)
      rc[i] = (i < (size_t)C) ? 0.f : kRefNegInf;
  }
  const int G = kKT / C;  // duration slots per label
  const int c = tid % C, ks = tid / C;
  const bool act = ks < G;
  // durations per chunk: all at once (forward, resident), else the x-row / staging chunk
  const int cs = (sp.resident && dir == 0) ? kcap : sp.kc;
  int par = 0;  // staging buffer holding the current chunk
  auto issue = [&](int k0, int nk, int q) {
    double* dst = ebuf + (size_t)q * sp.kc * cc;
    const double* src = Eg + (size_t)k0 * cc;
    const int n = nk * (int)cc;
    for (int i = tid; i < n; i += kKT) cp_async8(dst + i, src + i);
    cp_async_commit();
  };
  // E rows of duration k inside the current chunk starting at k0
  auto erow = [&](int k, int k0) -> const double* {
    return resident ? Eall + (size_t)k * cc
                    : ebuf + (size_t)par * sp.kc * cc + (size_t)(k - k0) * cc;
  };
  // before a chunk: queue the next one (of this or the next position), wait for this one
  auto stage = [&](int k0, int kmax, int tnext, int kmax_next) {
    if (resident) return;
    if (k0 + cs <= kmax)
      issue(k0 + cs, min(cs, kmax - (k0 + cs) + 1), par ^ 1);
    else if (tnext >= 0)
      issue(1, min(cs, kmax_next), par ^ 1);
    else
      cp_async_commit();
    cp_async_wait1();
  };

  // vals[] holds position t's log values: store them in the ring and tables
  auto finish = [&](int t) {
    const int slot = t % R;
    if (dir == 0) {
      if (warp == 0) {
        double mm = -INFINITY;
        for (int q = lane; q < C; q += 32) mm = fmax(mm, vals[q]);
        for (int o = 16; o > 0; o >>= 1) mm = fmax(mm, __shfl_xor_sync(0xffffffffu, mm, o));
        if (lane == 0) s_m = mm;
      }
      __syncthreads();
      const double m = s_m;
      for (int q = tid; q < C; q += kKT) {
        const double v = vals[q];
        ring[(size_t)slot * C + q] =
            SEMI == 0 ? ((m > -INFINITY && v > -INFINITY) ? exp(v - m) : 0.0) : v;
        if (use_rso) rso[(size_t)slot * C + q] = (SEMI == 0 ? m : 0.0) + dt[q];
        if (a.alpha) a.alpha[((size_t)b * (T + 1) + t) * C + q] = v;
        if (a.ref_ckpt) {
          const int S = a.sref;
          const int ic = (t + S - 1) / S;
          if (ic < a.nref && (long long)ic * S <= Lb && (long long)ic * S - t < K)
            a.ref_ckpt[(((size_t)b * a.nref + ic) * K + (t % K)) * C + q] =
                v > -INFINITY ? (float)v : kRefNegInf;
        }
      }
      if (tid == 0) {
        rn[slot] = m;
        if (a.amax) a.amax[(size_t)b * (T + 1) + t] = m;
      }
    } else {
      for (int q = tid; q < C; q += kKT) {
        const double v = vals[q];
        ring[(size_t)slot * C + q] = v > -INFINITY ? v + ct[q] : -INFINITY;
        if (a.beta) a.beta[((size_t)b * (T + 1) + t) * C + q] = v;
      }
    }
    __syncthreads();
  };
  // the G partial results of each label -> vals[label]: one warp per label,
  // a shuffle max, one exp per slot and a shuffle sum
  auto combine = [&](double m, double S) {
    redm[tid] = m;
    reds[tid] = S;
    __syncthreads();
    for (int lc = warp; lc < C; lc += kKT / 32) {
      double mm = -INFINITY;
      for (int j = lane; j < G; j += 32) mm = fmax(mm, redm[j * C + lc]);
      for (int o = 16; o > 0; o >>= 1) mm = fmax(mm, __shfl_xor_sync(0xffffffffu, mm, o));
      double r = mm;
      if (SEMI == 0 && mm > -INFINITY) {
        double ss = 0.0;
        for (int j = lane; j < G; j += 32) {
          const double mj = redm[j * C + lc];
          if (mj > -INFINITY) ss += reds[j * C + lc] * exp(mj - mm);
        }
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        r = mm + log(ss);
      }
      if (lane == 0) {
        if (dir == 0 && r > -INFINITY) r += ct[lc];
        vals[lc] = r;
      }
    }
    __syncthreads();
  };
  // a batch of up to four items: fold sum_u v_u exp(x_u) into (m, S) with one rescale
  auto add_batch = [&](double& m, double& S, double* xv, double* av) {
    double bm = m;
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (av[u] > 0.0) {
        if (av[u] < 1e-280) {  // too small to scale by exp(x - m) alone: move into x
          xv[u] += log(av[u]);
          av[u] = 1.0;
        }
        bm = fmax(bm, xv[u]);
      }
    if (!(bm > -INFINITY)) return;
    double ns = (m > -INFINITY) ? S * exp(m - bm) : 0.0;
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (av[u] > 0.0) ns += av[u] * exp(xv[u] - bm);
    S = ns;
    m = bm;
  };
  // dot product of a source row with column c of E[k] (stride C)
  auto dot = [&](const double* x, const double* e) {
    double a0 = 0.0, a1 = 0.0, a2 = 0.0, a3 = 0.0;
    int q = 0;
    for (; q + 3 < C; q += 4) {
      a0 = fma(x[q], e[(size_t)q * C], a0);
      a1 = fma(x[q + 1], e[(size_t)(q + 1) * C], a1);
      a2 = fma(x[q + 2], e[(size_t)(q + 2) * C], a2);
      a3 = fma(x[q + 3], e[(size_t)(q + 3) * C], a3);
    }
    for (; q < C; ++q) a0 = fma(x[q], e[(size_t)q * C], a0);
    return (a0 + a1) + (a2 + a3);
  };
  auto vmax = [&](const double* x, const double* e) {
    double mp = -INFINITY;
    for (int q = 0; q < C; ++q) mp = fmax(mp, x[q] + e[(size_t)q * C]);
    return mp;
  };
  // the per-position input terms, loaded before the position's items so their
  // latency hides behind them: dt = ps[t] - cum[t], ct = cum[t] + pe[t-1]
  auto load_terms = [&](int t) {
    for (int q = tid; q < C; q += kKT) {
      const double cv = cu(t, q);
      dt[q] = psv(t, q) - cv;
      ct[q] = cv + pev(t, q);
    }
  };

  for (int q = tid; q < C; q += kKT) vals[q] = 0.0;  // alpha[0] = 0, beta[len] = 0
  load_terms(dir == 0 ? 0 : Lb);
  __syncthreads();
  if (dir == 0) {
    finish(0);
    if (!resident && Lb >= 1) issue(1, 1, par);
    for (int t = 1; t <= Lb; ++t) {
      const int kmax = t < kcap ? t : kcap;
      const int tn = t + 1 <= Lb ? t + 1 : -1;
      const int kmax_n = tn > 0 ? (tn < kcap ? tn : kcap) : 0;
      load_terms(t);
      double m = -INFINITY, S = 0.0;
      for (int k0 = 1; k0 <= kmax; k0 += cs) {
        const int nk = min(cs, kmax - k0 + 1);
        stage(k0, kmax, tn, kmax_n);
        if (!resident) __syncthreads();
        if (act)
          for (int kb = ks; kb < nk; kb += 4 * G) {
            double xv[4], av[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const int kk = kb + u * G;
              xv[u] = -INFINITY;
              av[u] = 0.0;
              if (kk >= nk) continue;
              const int k = k0 + kk, s = t - k, slot = s % R;
              const double* src = ring + (size_t)slot * C;
              const double* e = erow(k, k0) + c;
              const double so = use_rso ? rso[(size_t)slot * C + c]
                                        : (SEMI == 0 ? rn[slot] : 0.0) + psv(s, c) - cu(s, c);
              if (SEMI == 0) {
                av[u] = dot(src, e);
                xv[u] = so + (double)t1f[k * C + c] + (double)dbf[k * C + c];
              } else {
                const double mp = vmax(src, e);
                if (mp > -INFINITY) m = fmax(m, mp + so);  // rf holds tr + db
              }
            }
            if (SEMI == 0) add_batch(m, S, xv, av);
          }
        if (!resident) {
          __syncthreads();
          par ^= 1;
        }
      }
      combine(m, S);
      finish(t);
    }
    if (tid == 0) {
      double lz = (double)kRefNegInf;
      if (Lb > 0) {
        double M = -INFINITY;
        for (int q = 0; q < C; ++q) M = fmax(M, vals[q]);
        if (M > -INFINITY) {
          lz = M;
          if (SEMI == 0) {
            double Sz = 0.0;
            for (int q = 0; q < C; ++q) Sz += exp(vals[q] - M);
            lz = M + log(Sz);
          }
        }
      }
      if (a.logz) a.logz[b] = lz;
      if (a.partition) a.partition[b] = (float)lz;
    }
  } else {
    finish(Lb);
    if (!resident && Lb >= 1) issue(1, 1, par);
    for (int t = Lb - 1; t >= 0; --t) {
      const int kmax = (Lb - t) < kcap ? (Lb - t) : kcap;
      const int tn = t - 1;
      const int kmax_n = tn >= 0 ? ((Lb - tn) < kcap ? (Lb - tn) : kcap) : 0;
      load_terms(t);
      __syncthreads();
      double m = -INFINITY, S = 0.0;
      for (int k0 = 1; k0 <= kmax; k0 += cs) {
        const int nkc = min(cs, kmax - k0 + 1);
        stage(k0, kmax, tn, kmax_n);
        // the source rows x[k][q] of this chunk of durations, all threads
        for (int i = tid; i < nkc * C; i += kKT) {
          const int kk = i / C, q = i % C, k = k0 + kk;
          // the max semiring's rb holds tr + db already
          xs[i] = ring[(size_t)((t + k) % R) * C + q] + (SEMI == 0 ? (double)dbf[k * C + q] : 0.0) +
                  dt[q];
        }
        __syncthreads();
        if (SEMI == 0) {
          // row maxima (one warp per row), then the rows in linear form
          for (int kk = warp; kk < nkc; kk += kKT / 32) {
            double mx = -INFINITY;
            for (int q = lane; q < C; q += 32) mx = fmax(mx, xs[kk * C + q]);
            for (int o = 16; o > 0; o >>= 1) mx = fmax(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            if (lane == 0) xm[kk] = mx;
          }
          __syncthreads();
          for (int i = tid; i < nkc * C; i += kKT) {
            const double mx = xm[i / C], x = xs[i];
            xs[i] = (mx > -INFINITY && x > -INFINITY) ? exp(x - mx) : 0.0;
          }
          __syncthreads();
        }
        if (act)
          for (int kb = ks; kb < nkc; kb += 4 * G) {
            double xv[4], av[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const int kk = kb + u * G;
              xv[u] = -INFINITY;
              av[u] = 0.0;
              if (kk >= nkc) continue;
              const int k = k0 + kk;
              const double* x = xs + kk * C;
              const double* e = erow(k, k0) + c;
              if (SEMI == 0) {
                if (xm[kk] > -INFINITY) {
                  av[u] = dot(x, e);
                  xv[u] = xm[kk] + (double)t1f[k * C + c];
                }
              } else {
                m = fmax(m, vmax(x, e));
              }
            }
            if (SEMI == 0) add_batch(m, S, xv, av);
          }
        __syncthreads();
        if (!resident) par ^= 1;
      }
      combine(m, S);
      finish(t);
    }
  }
}

// start term st[s,c] = amax[s] + ps[s,c] - cum[s,c] - logZ (s < len) and end
// term et[e,c] = beta[e,c] + cum[e,c] + pe[e-1,c] (1 <= e <= len); -inf elsewhere
__global__ void kcc_terms_kernel(const KccArgs a) {
  if (a.gate && *a.gate == 0) return;
  const int C = a.C, T = a.T;
  const size_t total = (size_t)a.B * (T + 1) * C;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const int c = (int)(i % C);
    const size_t bt = i / C;
    const int t = (int)(bt % (T + 1)), b = (int)(bt / (T + 1));
    const int Lb = seq_len(a.lengths, b, T);
    const double cum = (double)a.cum[i];
    double sv = -INFINITY, ev = -INFINITY;
    if (t < Lb) {
      const double n = a.amax[bt];
      if (n > -INFINITY)
        sv = n + (a.ps ? (double)a.ps[((size_t)b * T + t) * C + c] : 0.0) - cum - a.logz[b];
    }
    if (t >= 1 && t <= Lb) {
      const double bv = a.beta[i];
      if (bv > -INFINITY)
        ev = bv + cum + (a.pe ? (double)a.pe[((size_t)b * T + t - 1) * C + c] : 0.0);
    }
    a.st[i] = sv;
    a.et[i] = ev;
  }
}

// max semiring: the end marginal of every (position, label), summed over its
// incoming segments (the log semiring has it as exp(alpha + beta - logZ))
__global__ void kcc_pend_max_kernel(const KccArgs a) {
  if (a.gate && *a.gate == 0) return;
  const int C = a.C, T = a.T, kcap = a.kcap;
  const size_t total = (size_t)a.B * (T + 1) * C;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const int c = (int)(i % C);
    const size_t bt = i / C;
    const int e = (int)(bt % (T + 1)), b = (int)(bt / (T + 1));
    const double ev = a.et[i];
    double sum = 0.0;
    if (ev > -INFINITY) {
      const size_t row0 = (size_t)b * (T + 1);
      const int kmax = e < kcap ? e : kcap;
      for (int k = 1; k <= kmax; ++k) {
        const size_t s = row0 + e - k;
        const double sv = a.st[s * C + c];
        if (!(sv > -INFINITY)) continue;
        const double base = sv - a.amax[s] + ev + (double)a.db[k * C + c];
        const double* al = a.alpha + s * C;
        const float* tk = a.tr + (size_t)k * C * C + c;
        for (int q = 0; q < C; ++q) {
          const double x = al[q] + (double)tk[(size_t)q * C] + base;
          if (x > -INFINITY) sum += exp(x);
        }
      }
    }
    a.pend[i] = sum;
  }
}

struct PosPlan {
  int nsg, SB, kch, ef_smem;
  size_t al, st, ec, td, efs, total;  // offsets in doubles
};
__host__ __device__ inline PosPlan pos_plan(int C, int kcap) {
  PosPlan p{};
  p.nsg = kKT / C;
  p.SB = p.nsg * kJ;
  p.ef_smem = (size_t)C * C <= 8192;
  p.kch = p.ef_smem ? (int)(8192 / ((size_t)C * C)) : 4;
  if (p.kch > kcap) p.kch = kcap;
  if (p.kch < 1) p.kch = 1;
  size_t o = 0;
  p.al = o;
  o += (size_t)p.SB * C;
  p.st = o;
  o += (size_t)p.SB * C;
  p.ec = o;
  o += (size_t)(p.SB + p.kch - 1) * C;
  p.td = o;
  o += (size_t)p.kch * C;
  p.efs = o;
  if (p.ef_smem) o += (size_t)p.kch * C * C;
  p.total = o;
  return p;
}

// start marginals Pstart[s,c] = sum_{k,c'} P(s -> s+k, c' -> c) for a block of
// positions of one sequence; with the end marginals they give grad_cum,
// grad_proj_start and grad_proj_end.  Thread (label c, group g) owns the
// positions g + nsg*j, j < kJ, so each transition factor it loads serves kJ
// positions.
__global__ void __launch_bounds__(kKT) kcc_pos_kernel(const KccArgs a) {
  if (a.gate && *a.gate == 0) return;
  extern __shared__ __align__(16) double psm[];
  const int C = a.C, T = a.T, kcap = a.kcap;
  const PosPlan pp = pos_plan(C, kcap);
  const int b = blockIdx.y, s0 = blockIdx.x * pp.SB, tid = threadIdx.x;
  const int Lb = seq_len(a.lengths, b, T);
  double* al = psm + pp.al;
  double* sts = psm + pp.st;
  double* ec = psm + pp.ec;
  double* td = psm + pp.td;
  double* efs = psm + pp.efs;
  const size_t row0 = (size_t)b * (T + 1);
  for (int i = tid; i < pp.SB * C; i += kKT) {
    const int si = i / C, q = i % C, s = s0 + si;
    double av = 0.0, sv = -INFINITY;
    if (s < Lb) {
      const double n = a.amax[row0 + s];
      const double v = a.alpha[(row0 + s) * C + q];
      if (n > -INFINITY && v > -INFINITY) av = exp(v - n);
      sv = a.st[(row0 + s) * C + q];
    }
    al[i] = av;
    sts[i] = sv;
  }
  const int c = tid % C, sg = tid / C;
  const bool act = sg < pp.nsg;
  double acc[kJ];
#pragma unroll
  for (int j = 0; j < kJ; ++j) acc[j] = 0.0;
  const int kend = min(kcap, Lb - s0);  // no segment starting in this block is longer
  for (int k0 = 1; k0 <= kend; k0 += pp.kch) {
    const int nk = min(pp.kch, kend - k0 + 1);
    __syncthreads();
    for (int i = tid; i < (pp.SB + nk - 1) * C; i += kKT) {
      const int r = i / C, q = i % C, e = s0 + k0 + r;
      ec[i] = e <= Lb ? a.et[(row0 + e) * C + q] : -INFINITY;
    }
    for (int i = tid; i < nk * C; i += kKT) td[i] = a.pr.tdf[(size_t)k0 * C + i];
    if (pp.ef_smem)
      for (size_t i = tid; i < (size_t)nk * C * C; i += kKT)
        efs[i] = a.pr.ef[(size_t)k0 * C * C + i];
    __syncthreads();
    if (!act) continue;
    for (int kk = 0; kk < nk; ++kk) {
      const double* e =
          (pp.ef_smem ? efs + (size_t)kk * C * C : a.pr.ef + (size_t)(k0 + kk) * C * C) + c;
      double y[kJ];
#pragma unroll
      for (int j = 0; j < kJ; ++j) y[j] = 0.0;
      for (int q = 0; q < C; ++q) {
        const double ev = e[(size_t)q * C];
#pragma unroll
        for (int j = 0; j < kJ; ++j) y[j] = fma(al[(sg + pp.nsg * j) * C + q], ev, y[j]);
      }
#pragma unroll
      for (int j = 0; j < kJ; ++j) {
        const int si = sg + pp.nsg * j;
        const double x = sts[si * C + c] + ec[(si + kk) * C + c] + td[kk * C + c];
        if (x > -INFINITY) acc[j] = fma(y[j], exp(x), acc[j]);
      }
    }
  }
  if (!act) return;
  const double g = (double)a.grad_output[b];
  const double lz = a.logz[b];
#pragma unroll
  for (int j = 0; j < kJ; ++j) {
    const int s = s0 + sg + pp.nsg * j;
    if (s > T) continue;
    const size_t i = (row0 + s) * C + c;
    double pend = 0.0;
    if (s >= 1 && s <= Lb) {
      if (a.semiring == SEMICRF_MAX) {
        pend = a.pend[i];
      } else {
        const double v = a.alpha[i] + a.beta[i] - lz;
        pend = v > -INFINITY ? exp(v) : 0.0;
      }
    }
    const double pst = s < Lb ? acc[j] : 0.0;
    a.grad_cum[i] = (float)(g * (pend - pst));
    if (a.grad_ps && s < T) a.grad_ps[((size_t)b * T + s) * C + c] = (float)(g * pst);
    if (a.grad_pe && s >= 1) a.grad_pe[((size_t)b * T + s - 1) * C + c] = (float)(g * pend);
  }
}

// Transition marginals: part[slice][c'][(k-1)*C + c] = sum over the slice's
// positions s of g_b alpha_lin[s,c'] q[s,k,c], q = exp(st + tf + db + et).
// One CTA per (column tile, row tile, slice); each thread keeps a 4 x 8 tile
// of accumulators in registers.
__global__ void __launch_bounds__(kKT) kcc_tr_kernel(const KccArgs a) {
  if (a.gate && *a.gate == 0) return;
  const int C = a.C, T = a.T, kcap = a.kcap, B = a.B;
  const int ncol = kcap * C;
  const int col0 = blockIdx.x * kTC, r0 = blockIdx.y * kTR, slice = blockIdx.z;
  const int tid = threadIdx.x, tx = tid & 31, ty = tid >> 5;
  __shared__ double al[kTR];
  __shared__ double qv[kTC];
  double acc[4][8];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.0;
  // this thread's column of the q staging
  const int col = col0 + tid;
  const bool cv = col < ncol;
  const int kq = cv ? 1 + col / C : 1, cq = cv ? col % C : 0;
  const double tdq = cv ? a.pr.tdf[(size_t)kq * C + cq] : 0.0;
  const int nch = (2 * a.nslice + B - 1) / B;
  const int clen = (T + nch - 1) / nch;
  for (int u = slice; u < B * nch; u += a.nslice) {
    const int b = u / nch, ch = u % nch;
    const int Lb = seq_len(a.lengths, b, T);
    const int s_lo = ch * clen, s_hi = min((ch + 1) * clen, Lb);
    const size_t row0 = (size_t)b * (T + 1);
    const double g = (double)a.grad_output[b];
    for (int s = s_lo; s < s_hi; ++s) {
      __syncthreads();
      if (tid < kTR) {
        const int r = r0 + tid;
        double v = 0.0;
        if (r < C) {
          const double n = a.amax[row0 + s];
          const double x = a.alpha[(row0 + s) * C + r];
          if (n > -INFINITY && x > -INFINITY) v = exp(x - n);
        }
        al[tid] = v;
      }
      {
        double v = 0.0;
        const int e = s + kq;
        if (cv && e <= Lb) {
          const double x = a.st[(row0 + s) * C + cq] + tdq + a.et[(row0 + e) * C + cq];
          if (x > -INFINITY) v = g * exp(x);
        }
        qv[tid] = v;
      }
      __syncthreads();
      double ar[4], qr[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) ar[i] = al[ty + 8 * i];
#pragma unroll
      for (int j = 0; j < 8; ++j) qr[j] = qv[tx + 32 * j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fma(ar[i], qr[j], acc[i][j]);
    }
  }
  double* out = a.part_tr + (size_t)slice * C * ncol;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = r0 + ty + 8 * i;
    if (r >= C) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int cc = col0 + tx + 32 * j;
      if (cc < ncol) out[(size_t)r * ncol + cc] = acc[i][j];
    }
  }
}

// grad_tr[k][c'][c] = ef[k][c'][c] * sum_slice part; grad_db[k][c] = sum_c' grad_tr[k][c'][c]
__global__ void kcc_reduce_kernel(const KccArgs a, float* grad_tr, float* grad_db) {
  if (a.gate && *a.gate == 0) return;
  const int C = a.C, K = a.K, kcap = a.kcap;
  const int ncol = kcap * C;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < K * C; i += gridDim.x * blockDim.x) {
    const int k = i / C, c = i % C;
    double dsum = 0.0;
    for (int q = 0; q < C; ++q) {
      double v = 0.0;
      if (k >= 1 && k <= kcap) {
        const size_t j = (size_t)q * ncol + (size_t)(k - 1) * C + c;
        for (int sl = 0; sl < a.nslice; ++sl) v += a.part_tr[(size_t)sl * C * ncol + j];
        // the blocked kernels' partial sums carry the weights xf, the others ef
        v *= (a.al ? a.pr.xf : a.pr.ef)[((size_t)k * C + q) * C + c];
      }
      grad_tr[((size_t)k * C + q) * C + c] = (float)v;
      dsum += v;
    }
    grad_db[i] = (float)dsum;
  }
}

int grid_for(size_t n, int threads) {
  size_t g = (n + threads - 1) / threads;
  if (g > device_sm_count() * 16) g = device_sm_count() * 16;
  return g < 1 ? 1 : (int)g;
}

}  // namespace

bool kcc_supported(int C, int K) {
  if (K < 2 || C < 1 || C > kKT) return false;  // transition[k] is used for k = 1 .. K-1
  const ChainPlan cp = chain_plan(C, K);
  if (cp.kc < 1 || cp.total * 8 > kSmemMax) return false;
  return pos_plan(C, K - 1).total * 8 <= kSmemMax;
}

// both semirings: ef, eb, tf, tb, tdf and the blocked kernels' xf, xb, fk;
// the max semiring adds rf, rb
size_t kcc_prep_doubles(int K, int C, int semiring) {
  const size_t kcc = (size_t)K * C * C;
  return (semiring == SEMICRF_MAX ? 6 : 4) * kcc + 3 * (size_t)K * C + (size_t)C;
}

KccPrep kcc_prep_carve(double* base, int K, int C, int semiring) {
  KccPrep p{};
  if (!base) return p;
  const size_t kcc = (size_t)K * C * C, kc = (size_t)K * C;
  p.ef = base;
  p.eb = p.ef + kcc;
  p.tf = p.eb + kcc;
  p.tb = p.tf + kc;
  p.tdf = p.tb + kc;
  p.xf = p.tdf + kc;
  p.xb = p.xf + kcc;
  p.fk = p.xb + kcc;
  if (semiring == SEMICRF_MAX) {
    p.rf = p.fk + C;
    p.rb = p.rf + kcc;
  }
  return p;
}

int kcc_tr_slices(int B, int K, int C) {
  const int kcap = K - 1;
  const int tiles = ((kcap * C + kTC - 1) / kTC) * ((C + kTR - 1) / kTR);
  int ns = (2 * device_sm_count() + tiles - 1) / tiles;
  const int bmax = 4 * (B > 0 ? B : 1);
  if (ns > bmax) ns = bmax;
  return ns < 1 ? 1 : ns;
}

// the raw factors rf / rb are written when the carve gave them (max semiring)
cudaError_t launch_kcc_prep(const float* tr, const float* db, int K, int C, const KccPrep& pr,
                            cudaStream_t s) {
  kcc_prep_kernel<<<grid_for((size_t)K * C, 128), 128, 0, s>>>(tr, db, K, C, pr);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  return launch_kblk_prep(tr, db, K, C, pr, s);  // the blocked chain's weights (log semiring)
}

cudaError_t launch_kcc_chains(const KccArgs& a0, int ndir, cudaStream_t s) {
  if (a0.B <= 0) return cudaSuccess;
  KccArgs a = a0;
  const bool have = a.semiring == SEMICRF_MAX ? (a.pr.rf != nullptr) : (a.pr.xf != nullptr);
  if (have && kblk_supported(a.C, a.K)) {
    const bool guard = a.semiring == SEMICRF_LOG && a.kflag;
    if (guard) {
      cudaError_t e = cudaMemsetAsync(a.kflag, 0, sizeof(int), s);
      if (e != cudaSuccess) return e;
    }
    cudaError_t e = launch_kblk_chains(a, ndir, s);
    if (e != cudaSuccess || !guard) return e;
    // the log chain's float64 factors left their range (very large emission
    // scores): the per-position chain below redoes the tables in the log
    // domain; otherwise it returns at once
    a.gate = a.kflag;
    a.kflag = nullptr;
  }
  const size_t bytes = chain_plan(a.C, a.K).total * 8;
  auto go = [&](auto kern) -> cudaError_t {
    cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e != cudaSuccess) return e;
    kern<<<dim3(a.B, ndir), kKT, bytes, s>>>(a);
    return cudaGetLastError();
  };
  return a.semiring == SEMICRF_LOG ? go(kcc_chain_kernel<0>) : go(kcc_chain_kernel<1>);
}

cudaError_t launch_kcc_grads(const KccArgs& a, float* grad_tr, float* grad_db, cudaStream_t s) {
  if (a.B <= 0) return cudaSuccess;
  const size_t n = (size_t)a.B * (a.T + 1) * a.C;
  kcc_terms_kernel<<<grid_for(n, 256), 256, 0, s>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  if (a.al) {  // blocked kernels (kblk.cu), both semirings
    e = launch_kblk_grads(a, s);
    if (e != cudaSuccess) return e;
    kcc_reduce_kernel<<<grid_for((size_t)a.K * a.C, 128), 128, 0, s>>>(a, grad_tr, grad_db);
    e = cudaGetLastError();
    if (e != cudaSuccess || !a.kflag) return e;
    // fallback: when the blocked factors left the float64 range (very large
    // emission scores) the per-item kernels below redo every gradient in the log
    // domain; otherwise each of them returns at once
    KccArgs f = a;
    f.al = nullptr;
    f.anc = nullptr;
    f.ep1 = nullptr;
    f.gate = a.kflag;
    f.kflag = nullptr;
    f.nslice = kcc_tr_slices(a.B, a.K, a.C);
    return launch_kcc_grads(f, grad_tr, grad_db, s);
  }
  if (a.semiring == SEMICRF_MAX) {
    kcc_pend_max_kernel<<<grid_for(n, 128), 128, 0, s>>>(a);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  const PosPlan pp = pos_plan(a.C, a.kcap);
  const size_t pbytes = pp.total * 8;
  e = cudaFuncSetAttribute(kcc_pos_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)pbytes);
  if (e != cudaSuccess) return e;
  kcc_pos_kernel<<<dim3((a.T + 1 + pp.SB - 1) / pp.SB, a.B), kKT, pbytes, s>>>(a);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const int ncol = a.kcap * a.C;
  kcc_tr_kernel<<<dim3((ncol + kTC - 1) / kTC, (a.C + kTR - 1) / kTR, a.nslice), kKT, 0, s>>>(a);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  kcc_reduce_kernel<<<grid_for((size_t)a.K * a.C, 128), 128, 0, s>>>(a, grad_tr, grad_db);
  return cudaGetLastError();
}

}  // namespace semicrf
