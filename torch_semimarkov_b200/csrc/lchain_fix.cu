// lchain_fix.cu -- the log-domain fallback of the (C, C) log-semiring chain.
//
// lchain_ws_kernel keeps float64 linear values relative to per-block frames;
// when the scores inside one of its 8-position blocks span more than the
// float64 exponent range (emission scores of hundreds of log-units per block),
// one of its exponent clamps clips and it sets the launch's overflow flag.
// This kernel, launched right after it, then recomputes the same chains in the
// log domain and overwrites their outputs; with the flag clear it returns at
// once.  In the chain's own position index u (u = t forward, u = len - t
// backward; the recurrence of pytorch_reference.py:116-273 and :276-525):
//   x[u,c] = toff(u,c) + s cum(u,c) + LSE_{k=1..min(u,kcap)} ( v[u-k,c] + db[k,c] )
//   v[u,c] = m[u,c] + soff(u,c) - s cum(u,c),   m[u,c] = LSE_c' ( x[u,c'] + M[c',c] )
// with s = +1 forward (x = alpha, m = A, M = transition) and s = -1 backward
// (x = G, m = beta, M = transition^T), and the start rows alpha[0] = 0 and
// beta[len] = 0.  The m row is formed from the prepared exp(M - colmax) as
// m[c] = xmax + colmax[c] + log sum_c' exp(x[c'] - xmax) exp(M[c',c] - colmax[c]),
// with a per-term log-domain sum for a column whose products all underflow;
// exp(M - colmax) is staged in shared memory when C * C doubles fit beside the
// ring and read from global memory otherwise (C up to 256).  db comes from the
// prepared log duration table.  The rows written are the chain tables
// a = exp(x - n), A = exp(m - n) and n (n = the row's largest x or m), and log Z
// = LSE_c alpha[len, c], exactly what the backward reads; for a forward that
// also returns the reference's ring checkpoints (launch_streaming_triton_kernel
// layout, (B, nref, K, C) float32 log alpha) the rows inside each checkpoint's
// window are rewritten too.

#include "semicrf_internal.cuh"

namespace semicrf {

namespace {

constexpr int kFT = 256;
constexpr size_t kFSmemMax = 200 * 1024;

// the ring, the row vectors and the reduction scratch; plus C * C when M is staged
__host__ __device__ inline size_t fix_smem_doubles(int C, int K, bool stage_m) {
  const int kcap = K - 1 > 1 ? K - 1 : 1;
  return (size_t)kcap * C + (stage_m ? (size_t)C * C : 0) + 4 * (size_t)C + 2 * kFT + 8;
}

inline bool fix_stage_m(int C, int K) { return fix_smem_doubles(C, K, true) * 8 <= kFSmemMax; }

__global__ void __launch_bounds__(kFT) lchain_fix_kernel(const LChainLaunch L, int stage_m) {
  if (!L.ovf || *L.ovf == 0) return;
  extern __shared__ __align__(16) double fsm[];
  const int C = L.C, K = L.K, T = L.T;
  const int kcap = K - 1 > 1 ? K - 1 : 1;
  const int ci = blockIdx.x, tid = threadIdx.x;
  const bool second = ci >= L.n1;
  const LChainArgs& A = second ? L.a1 : L.a0;
  const int b = second ? ci - L.n1 : ci;
  if (b >= L.B) return;
  const int dir = A.dir;
  const double sg = dir == 0 ? 1.0 : -1.0;
  const long long lraw = A.lengths[b];
  const int Lb = lraw < 0 ? 0 : (lraw > T ? T : (int)lraw);
  double* ring = fsm;                                // [kcap][C]: v of the last kcap positions
  double* Ms = ring + (size_t)kcap * C;              // [C][C]: exp(M - colmax), when staged
  double* xr = Ms + (stage_m ? (size_t)C * C : 0);   // [C]
  double* er = xr + C;                               // [C]: exp(x - xmax)
  double* mr = er + C;                               // [C]
  double* pm = mr + 2 * C;                           // [kFT] partial maxima
  double* ps2 = pm + kFT;                            // [kFT] partial sums
  double* nrow = ps2 + kFT;                          // [2]: n, xmax
  const double* Mg = stage_m ? Ms : A.mx;
  const float* cum_b = A.cum + (size_t)b * (T + 1) * C;
  const float* ps_b = A.ps ? A.ps + (size_t)b * T * C : nullptr;
  const float* pe_b = A.pe ? A.pe + (size_t)b * T * C : nullptr;
  auto cpos = [&](int u) { return dir == 0 ? u : Lb - u; };
  auto soff = [&](int u, int c) -> double {
    const int t = cpos(u);
    if (dir == 0) return (ps_b && t < T) ? (double)ps_b[(size_t)t * C + c] : 0.0;
    return (pe_b && t >= 1) ? (double)pe_b[(size_t)(t - 1) * C + c] : 0.0;
  };
  auto toff = [&](int u, int c) -> double {
    const int t = cpos(u);
    if (dir == 0) return (pe_b && t >= 1) ? (double)pe_b[(size_t)(t - 1) * C + c] : 0.0;
    return (ps_b && t < T) ? (double)ps_b[(size_t)t * C + c] : 0.0;
  };
  auto cumd = [&](int u, int c) -> double { return (double)cum_b[(size_t)cpos(u) * C + c]; };
  if (stage_m)
    for (int i = tid; i < C * C; i += kFT) Ms[i] = A.mx[i];
  double* atab = A.a_tab ? A.a_tab + (size_t)b * (T + 1) * C : nullptr;
  double* Atab = A.A_tab ? A.A_tab + (size_t)b * (T + 1) * C : nullptr;
  double* ntab = A.n_tab ? A.n_tab + (size_t)b * (T + 1) : nullptr;
  __syncthreads();
  // the row's m from its x, its tables, and its v into the ring
  auto finish_row = [&](int u) {
    if (tid == 0) {
      double xm = -INFINITY;
      for (int c = 0; c < C; ++c) xm = fmax(xm, xr[c]);
      nrow[1] = xm;
    }
    __syncthreads();
    const double xm = nrow[1];
    for (int q = tid; q < C; q += kFT) er[q] = xr[q] > -INFINITY ? exp(xr[q] - xm) : 0.0;
    __syncthreads();
    for (int c = tid; c < C; c += kFT) {
      double sm = 0.0;
      for (int q = 0; q < C; ++q) sm = fma(er[q], Mg[(size_t)q * C + c], sm);
      double m = -INFINITY;
      if (sm > 0.0) {
        m = xm + (double)A.colmax[c] + log(sm);
      } else if (xm > -INFINITY) {
        // every product underflowed: the same sum term by term in the log domain
        double mx = -INFINITY;
        for (int q = 0; q < C; ++q) {
          const double e = Mg[(size_t)q * C + c];
          if (e > 0.0 && xr[q] > -INFINITY) mx = fmax(mx, xr[q] + log(e));
        }
        if (mx > -INFINITY) {
          double s2 = 0.0;
          for (int q = 0; q < C; ++q) {
            const double e = Mg[(size_t)q * C + c];
            if (e > 0.0 && xr[q] > -INFINITY) s2 += exp(xr[q] + log(e) - mx);
          }
          m = mx + log(s2) + (double)A.colmax[c];
        }
      }
      mr[c] = m;
    }
    if (u == 0 && dir == 1)
      for (int c = tid; c < C; c += kFT) mr[c] = 0.0;  // beta[len] = 0
    __syncthreads();
    if (tid == 0) {
      double n = -INFINITY;
      for (int c = 0; c < C; ++c) n = fmax(n, fmax(xr[c], mr[c]));
      nrow[0] = n > -INFINITY ? n : 0.0;
    }
    __syncthreads();
    const double n = nrow[0];
    const int t = cpos(u);
    for (int c = tid; c < C; c += kFT) {
      if (atab) atab[(size_t)t * C + c] = xr[c] > -INFINITY ? exp(xr[c] - n) : 0.0;
      if (Atab) Atab[(size_t)t * C + c] = mr[c] > -INFINITY ? exp(mr[c] - n) : 0.0;
      ring[(size_t)(u % kcap) * C + c] =
          mr[c] > -INFINITY ? mr[c] + soff(u, c) - sg * cumd(u, c) : -INFINITY;
    }
    if (tid == 0 && ntab) ntab[t] = n;
    __syncthreads();
  };
  // start row: alpha[0] = 0 (forward); G[len] has no segment (backward)
  for (int c = tid; c < C; c += kFT) xr[c] = dir == 0 ? 0.0 : -INFINITY;
  __syncthreads();
  finish_row(0);
  // label c, duration slot j = tid / C of G slots
  const int G = kFT / C, c = tid % C, j = tid / C;
  for (int u = 1; u <= Lb; ++u) {
    const int kmax = u < kcap ? u : kcap;
    double m = -INFINITY, S = 0.0;
    if (j < G)
      for (int k = 1 + j; k <= kmax; k += G) {
        const double z = ring[(size_t)((u - k) % kcap) * C + c] +
                         (double)L.dbl[(size_t)k * C + c];
        if (!(z > -INFINITY)) continue;
        if (z > m) {
          S = S * exp(m - z) + 1.0;
          m = z;
        } else {
          S += exp(z - m);
        }
      }
    pm[tid] = m;
    ps2[tid] = S;
    __syncthreads();
    for (int cc = tid; cc < C; cc += kFT) {
      double mm = -INFINITY;
      for (int g = 0; g < G; ++g) mm = fmax(mm, pm[g * C + cc]);
      double ss = 0.0;
      if (mm > -INFINITY)
        for (int g = 0; g < G; ++g)
          if (pm[g * C + cc] > -INFINITY) ss += ps2[g * C + cc] * exp(pm[g * C + cc] - mm);
      xr[cc] = mm > -INFINITY ? toff(u, cc) + sg * cumd(u, cc) + mm + log(ss) : -INFINITY;
    }
    __syncthreads();
    if (dir == 0 && A.ref_ckpt) {
      // checkpoint ic holds alpha of the positions (ic S - K, ic S], slot u % K
      const int Sr = A.sref, ic = (u + Sr - 1) / Sr;
      if (ic < A.nref && ic * Sr <= Lb && ic * Sr - u < K)
        for (int cc = tid; cc < C; cc += kFT)
          A.ref_ckpt[(((size_t)b * A.nref + ic) * K + (u % K)) * C + cc] =
              xr[cc] > -INFINITY ? (float)xr[cc] : kRefNegInf;
    }
    finish_row(u);
  }
  if (dir == 0 && tid == 0) {
    double M = -INFINITY;
    for (int q = 0; q < C; ++q) M = fmax(M, xr[q]);
    double lz = (double)kRefNegInf;
    if (Lb > 0 && M > -INFINITY) {
      double Sz = 0.0;
      for (int q = 0; q < C; ++q) Sz += exp(xr[q] - M);
      lz = M + log(Sz);
    }
    if (A.partition) A.partition[b] = (float)lz;
    if (A.logz) A.logz[b] = lz;
  }
}

}  // namespace

bool lchain_fix_supported(int C, int K) {
  return C <= kFT && fix_smem_doubles(C, K, false) * 8 <= kFSmemMax;
}

cudaError_t launch_lchain_fix(const LChainLaunch& L, int grid, cudaStream_t s) {
  if (!L.ovf || grid <= 0) return cudaSuccess;
  const bool stage = fix_stage_m(L.C, L.K);
  const size_t bytes = fix_smem_doubles(L.C, L.K, stage) * 8;
  cudaError_t e = cudaFuncSetAttribute(lchain_fix_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e != cudaSuccess) return e;
  lchain_fix_kernel<<<grid, kFT, bytes, s>>>(L, stage ? 1 : 0);
  return cudaGetLastError();
}

}  // namespace semicrf
