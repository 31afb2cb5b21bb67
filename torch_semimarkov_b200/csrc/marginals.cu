// marginals.cu -- gradients of the streaming semi-CRF from alpha/beta tables.
//
// Reference: streaming/pytorch_reference.py:425-499 accumulates, for every
// segment (t, k, c_dst, c_src), the marginal
//     m = exp(alpha[t,c_src] + edge + beta[t+k,c_dst] - logZ)
// into grad_cum[t+k] (+), grad_cum[t] (-), grad_tr, grad_db[min(k,K-1)] and
// grad_proj.  Summed over c_src and k these become per-position quantities
//     Pend[p,c]   = sum over segments with label c ending at p
//     Pstart[p,c] = sum over segments with label c starting at p
// so grad_cum[p,c] = Pend - Pstart, grad_ps[p,c] = Pstart, grad_pe[p-1,c] =
// Pend.  In the log semiring they have closed forms
//     Pend[p,c]   = exp(alpha[p,c] + beta[p,c] - logZ)
//     Pstart[p,c] = exp(A[p,c] + G[p,c] - logZ)
// with A, G the chain intermediates (see chain.cu).  The reference's max
// semiring keeps the same exp-sum marginals over max-semiring alpha/beta
// (:458-499); there A is replaced by A_lse = LSE_c'(alpha + tr) and Pend /
// Pstart are evaluated as explicit sums over k.
//   grad_tr[c',c] = sum_t exp(alpha[t,c'] + tr[c',c] - A_lse[t,c]) * Pstart[t,c]
//   grad_db[k,c]  = sum_t M[t,k,c]
//   M[t,k,c] = exp(A_lse[t,c] + ps[t,c] + cum[t+k,c] - cum[t,c] + pe[t+k-1,c]
//                  + beta[t+k,c] + db[k,c] - logZ)
// Per-sequence sums are accumulated in float64 by one thread per output
// element (no atomics) and reduced over the batch with grad_output weights.

#include "semicrf_internal.cuh"

namespace semicrf {

// A_lse[t,c] = LSE_c'(xa[t,c'] + tr[c',c]) relative to the same normaliser
// as xa (max semiring only; in the log semiring the chain's m table is it).
__global__ void alse_kernel(int B, int T, int C, const float* __restrict__ tr,
                            const int64_t* __restrict__ lengths, const float* __restrict__ xa,
                            float* __restrict__ alse) {
  const size_t total = (size_t)B * (T + 1) * C;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const int c = (int)(i % C);
    const size_t bt = i / C;
    const int t = (int)(bt % (T + 1));
    const int b = (int)(bt / (T + 1));
    long long lr = lengths[b];
    const int L = lr < 0 ? 0 : (lr > T ? T : (int)lr);
    if (t > L) {
      alse[i] = kNegInf;
      continue;
    }
    const float* x = xa + bt * C;
    float m = kNegInf;
    for (int q = 0; q < C; ++q) m = fmaxf(m, x[q] + tr[q * C + c]);
    float s = 0.f;
    if (m != kNegInf)
      for (int q = 0; q < C; ++q) s += __expf(x[q] + tr[q * C + c] - m);
    alse[i] = (m == kNegInf) ? kNegInf : m + __logf(s);
  }
}

__device__ __forceinline__ int clampL(long long l, int T) { return l < 0 ? 0 : (l > T ? T : (int)l); }

// M[t,k,c] for one (t, s = t+k, c); returns 0 outside the valid range.
__device__ __forceinline__ float seg_marginal(const MargArgs& a, const float* atab, int b, int L,
                                              int t, int k, int c) {
  const int s = t + k;
  if (t < 0 || s > L || k < 1 || k > a.kcap) return 0.f;
  const int T = a.T, C = a.C;
  const size_t rt = ((size_t)b * (T + 1) + t) * C + c;
  const size_t rs = ((size_t)b * (T + 1) + s) * C + c;
  const float av = atab[rt];
  const float bv = a.mb[rs];
  if (av == kNegInf || bv == kNegInf) return 0.f;
  const float dv = a.dbl[(size_t)k * C + c];
  if (dv == kNegInf) return 0.f;
  float small = av + bv + dv;
  if (a.ps) small += a.ps[((size_t)b * T + t) * C + c];
  if (a.pe) small += a.pe[((size_t)b * T + (s - 1)) * C + c];
  const double big = (a.na[(size_t)b * (T + 1) + t] + a.nb[(size_t)b * (T + 1) + s] - a.logz[b]) +
                     ((double)a.cum[rs] - (double)a.cum[rt]);
  return __expf((float)(big + (double)small));
}

// grad_cum / grad_ps / grad_pe and the Pstart table.
__global__ void pos_kernel(MargArgs a, const float* __restrict__ atab, int semiring,
                           float* __restrict__ pstart) {
  const int T = a.T, C = a.C;
  const size_t total = (size_t)a.B * (T + 1) * C;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const int c = (int)(i % C);
    const size_t bt = i / C;
    const int t = (int)(bt % (T + 1));
    const int b = (int)(bt / (T + 1));
    const int L = clampL(a.lengths[b], T);
    const double off = a.na[bt] + a.nb[bt] - a.logz[b];
    float pend = 0.f, pst = 0.f;
    if (semiring == 0) {
      if (t >= 1 && t <= L) pend = __expf((float)((double)(a.xa[i] + a.mb[i]) + off));
      if (t <= L - 1) pst = __expf((float)((double)(a.ma[i] + a.xb[i]) + off));
    } else {
      const int kc = a.kcap;
      for (int k = 1; k <= kc; ++k) {
        if (t - k >= 0 && t <= L) pend += seg_marginal(a, atab, b, L, t - k, k, c);
        if (t + k <= L) pst += seg_marginal(a, atab, b, L, t, k, c);
      }
    }
    if (!(pend == pend)) pend = 0.f;
    if (!(pst == pst)) pst = 0.f;
    const float g = a.grad_output[b];
    a.grad_cum[i] = g * (pend - pst);
    pstart[i] = pst;
    if (a.grad_ps && t < T) a.grad_ps[((size_t)b * T + t) * C + c] = g * pst;
    if (a.grad_pe && t >= 1) a.grad_pe[((size_t)b * T + (t - 1)) * C + c] = g * pend;
  }
}

// per-sequence transition gradient: one thread per (c', c) pair.
__global__ void tr_kernel(MargArgs a, const float* __restrict__ atab,
                          const float* __restrict__ pstart) {
  const int b = blockIdx.y;
  const int p = blockIdx.x * blockDim.x + threadIdx.x;
  const int T = a.T, C = a.C;
  if (p >= C * C) return;
  const int cs = p / C, cd = p % C;
  const int L = clampL(a.lengths[b], T);
  const float trv = a.tr[p];
  double acc = 0.0;
  if (trv != kNegInf) {
    for (int t = 0; t < L; ++t) {
      const size_t row = ((size_t)b * (T + 1) + t) * C;
      const float ps = pstart[row + cd];
      if (ps == 0.f) continue;
      const float w = __expf(a.xa[row + cs] + trv - atab[row + cd]);
      acc += (double)(w * ps);
    }
  }
  a.part_tr[(size_t)b * C * C + p] = (float)acc;
}

// per-sequence duration-bias gradient: one thread per (k, c).
__global__ void db_kernel(MargArgs a, const float* __restrict__ atab) {
  const int b = blockIdx.y;
  const int q = blockIdx.x * blockDim.x + threadIdx.x;
  const int T = a.T, C = a.C, K = a.K;
  const int L = clampL(a.lengths[b], T);
  float* out = a.part_db + (size_t)b * K * C;
  if (q < C && K > 1) out[q] = 0.f;  // row 0 is unused unless K == 1
  if (q >= a.kcap * C) return;
  const int k = q / C + 1, c = q % C;
  double acc = 0.0;
  for (int t = 0; t + k <= L; ++t) acc += (double)seg_marginal(a, atab, b, L, t, k, c);
  const int di = k < K - 1 ? k : K - 1;
  out[(size_t)di * C + c] = (float)acc;
}

__global__ void reduce_kernel(int B, int n, const float* __restrict__ part,
                              const float* __restrict__ g, float* __restrict__ out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  double acc = 0.0;
  for (int b = 0; b < B; ++b) acc += (double)g[b] * (double)part[(size_t)b * n + i];
  out[i] = (float)acc;
}

static int grid_for(size_t n, int bs) {
  size_t g = (n + bs - 1) / bs;
  if (g > device_sm_count() * 16) g = device_sm_count() * 16;
  if (g < 1) g = 1;
  return (int)g;
}

// semiring: 0 log, 1 max.  `alse` (B,T+1,C) is scratch for the max semiring;
// `pstart` (B,T+1,C) scratch for both.
cudaError_t launch_marginals_impl(const MargArgs& a, int semiring, float* alse, float* pstart,
                                  cudaStream_t s) {
  const size_t n = (size_t)a.B * (a.T + 1) * a.C;
  const float* atab = a.ma;
  if (semiring == 1) {
    alse_kernel<<<grid_for(n, 256), 256, 0, s>>>(a.B, a.T, a.C, a.tr, a.lengths, a.xa, alse);
    atab = alse;
  }
  pos_kernel<<<grid_for(n, 256), 256, 0, s>>>(a, atab, semiring, pstart);
  dim3 gt((a.C * a.C + 255) / 256, a.B);
  tr_kernel<<<gt, 256, 0, s>>>(a, atab, pstart);
  dim3 gd((a.kcap * a.C + 255) / 256 > (a.C + 255) / 256 ? (a.kcap * a.C + 255) / 256
                                                         : (a.C + 255) / 256,
          a.B);
  db_kernel<<<gd, 256, 0, s>>>(a, atab);
  return cudaGetLastError();
}

cudaError_t launch_reduce_shared(const MargArgs& a, float* grad_tr, float* grad_db,
                                 cudaStream_t s) {
  const int ntr = a.C * a.C, ndb = a.K * a.C;
  reduce_kernel<<<(ntr + 255) / 256, 256, 0, s>>>(a.B, ntr, a.part_tr, a.grad_output, grad_tr);
  reduce_kernel<<<(ndb + 255) / 256, 256, 0, s>>>(a.B, ndb, a.part_db, a.grad_output, grad_db);
  return cudaGetLastError();
}

}  // namespace semicrf
