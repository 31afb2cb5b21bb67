// escan.cu -- the edge-tensor scan (triton_scan.py of the reference).
//
// Input: log potentials edge (B, N-1, K, C, C), edge[b, s, j, c, c'] for a
// segment that starts at position s with duration index j, new label c and
// previous label c'.  The scan (triton_scan.py:163-273):
//   beta[0, c] = 0
//   beta[n, c] = (+)_{k=1..k_eff(n)} (+)_{c'} ( beta[n-k, c'] + edge[n-k, min(k, K-1), c, c'] )
//   k_eff(n)   = max(1, min(K-1, n))       (K = 1 still uses duration 1, edge index 0)
//   partition  = (+)_c beta[L-1, c]          (L = length; L = 1 gives (+) of zeros)
// with (+) = logsumexp or max; lengths 0 or > N leave the reference's -1e9.
// Gradients (the reference differentiates its PyTorch scan with autograd):
//   log: d partition / d edge[s, j, c, c'] = exp(beta[s,c'] + edge + gamma[s+k, c] - logZ)
//        for the duration k of index j, s + k <= L-1, with the outside values
//        gamma[L-1, .] = 0, gamma[s, c'] = (+)_{k,c} (edge[s, j(k), c, c'] + gamma[s+k, c]);
//   max: 1 on the edges of the first-maximum path (torch.max routes its
//        gradient to the first maximal index: first c', then smallest k, then
//        first final label), 0 elsewhere.
// Arithmetic is float64.  One CTA per sequence runs each chain; the log
// gradient is one parallel pass over the edge tensor in its own layout.

#include "semicrf_internal.cuh"

namespace semicrf {

namespace {

constexpr int kET = 256;

__device__ __forceinline__ int es_len(const int64_t* lengths, int b) {
  const long long l = lengths[b];
  return l < 0 ? 0 : (l > (1LL << 30) ? (1 << 30) : (int)l);
}

// shared memory of a chain CTA, in doubles: ring [K][C], item values
// [kcap][C] and (forward, max) the items' source-label argmax [kcap][C] ints
__host__ __device__ inline size_t es_smem(int K, int C) {
  const size_t kcap = K > 1 ? K - 1 : 1;
  return (size_t)K * C + kcap * C + (kcap * C + 1) / 2 + 8;
}

// Forward chain.  beta_tab (B, N, C) and the max semiring's backpointers
// (B, N, C) are written when given.
template <int SEMI>
__global__ void __launch_bounds__(kET) escan_fwd_kernel(int N, int K, int C, const float* edge,
                                                        const int64_t* lengths, float* partition,
                                                        double* logz, double* beta_tab,
                                                        int32_t* bp) {
  extern __shared__ __align__(16) double esm[];
  const int b = blockIdx.x, tid = threadIdx.x;
  const int L = es_len(lengths, b);
  const int R = K;  // ring: beta[n] in slot n % K
  const int kcap = K > 1 ? K - 1 : 1;
  double* ring = esm;                                              // [K][C]
  double* item = esm + (size_t)K * C;                              // [kcap][C]
  int* argbuf = reinterpret_cast<int*>(item + (size_t)kcap * C);  // [kcap][C]
  const size_t cc = (size_t)C * C;
  const float* edge_b = edge + (size_t)b * (N > 1 ? N - 1 : 0) * K * cc;
  // positions needed: 0 .. L-1 (the scan beyond L-1 does not reach the result)
  const int nlast = (L >= 1 && L <= N) ? L - 1 : -1;
  for (int c = tid; c < C; c += kET) {
    ring[c] = 0.0;
    if (beta_tab) beta_tab[(size_t)b * N * C + c] = 0.0;
  }
  __syncthreads();
  for (int n = 1; n <= nlast; ++n) {
    const int keff = n < kcap ? n : kcap;
    for (int it = tid; it < keff * C; it += kET) {
      const int k = 1 + it / C, c = it % C;
      const int s = n - k;
      const int j = k < K - 1 ? k : K - 1;
      const double* src = ring + (size_t)(s % R) * C;
      const float* e = edge_b + ((size_t)s * K + j) * cc + (size_t)c * C;
      double m = -INFINITY;
      int arg = 0;
      for (int q = 0; q < C; ++q) {
        const double v = src[q] + (double)e[q];
        if (v > m) {  // strict: the first maximal source label
          m = v;
          arg = q;
        }
      }
      double r = m;
      if (SEMI == 0 && m > -INFINITY) {
        double sum = 0.0;
        for (int q = 0; q < C; ++q) sum += exp(src[q] + (double)e[q] - m);
        r = m + log(sum);
      }
      item[(size_t)(k - 1) * C + c] = r;
      if (SEMI == 1) argbuf[(size_t)(k - 1) * C + c] = arg;
    }
    __syncthreads();
    for (int c = tid; c < C; c += kET) {
      double m = -INFINITY;
      int bk = 1;
      for (int k = 1; k <= keff; ++k) {
        const double v = item[(size_t)(k - 1) * C + c];
        if (v > m) {  // strict: the smallest maximising duration
          m = v;
          bk = k;
        }
      }
      double r = m;
      if (SEMI == 0 && m > -INFINITY) {
        double sum = 0.0;
        for (int k = 1; k <= keff; ++k) sum += exp(item[(size_t)(k - 1) * C + c] - m);
        r = m + log(sum);
      }
      ring[(size_t)(n % R) * C + c] = r;
      if (beta_tab) beta_tab[((size_t)b * N + n) * C + c] = r;
      if (SEMI == 1 && bp) bp[((size_t)b * N + n) * C + c] = bk | (argbuf[(size_t)(bk - 1) * C + c] << 16);
    }
    __syncthreads();
  }
  if (tid == 0) {
    double lz = (double)kRefNegInf;
    if (nlast >= 0) {
      const double* fin = ring + (size_t)(nlast % R) * C;
      double m = -INFINITY;
      for (int c = 0; c < C; ++c) m = fmax(m, fin[c]);
      lz = m;
      if (SEMI == 0 && m > -INFINITY) {
        double sum = 0.0;
        for (int c = 0; c < C; ++c) sum += exp(fin[c] - m);
        lz = m + log(sum);
      }
    }
    if (partition) partition[b] = (float)lz;
    if (logz) logz[b] = lz;
  }
}

// Outside chain (log semiring): gamma (B, N, C) for positions L-1 down to 0.
__global__ void __launch_bounds__(kET) escan_out_kernel(int N, int K, int C, const float* edge,
                                                        const int64_t* lengths, double* gamma) {
  extern __shared__ __align__(16) double esm[];
  const int b = blockIdx.x, tid = threadIdx.x;
  const int L = es_len(lengths, b);
  if (L < 1 || L > N) return;
  const int kcap = K > 1 ? K - 1 : 1;
  const size_t cc = (size_t)C * C;
  const float* edge_b = edge + (size_t)b * (N - 1) * K * cc;
  double* item = esm;  // [kcap][C]
  double* g_b = gamma + (size_t)b * N * C;
  for (int c = tid; c < C; c += kET) g_b[(size_t)(L - 1) * C + c] = 0.0;
  __syncthreads();
  for (int s = L - 2; s >= 0; --s) {
    const int kmax = (L - 1 - s) < kcap ? (L - 1 - s) : kcap;
    // item (k, c'): (+)_c edge[s, j, c, c'] + gamma[s+k, c]; consecutive
    // threads take consecutive c', so each c step reads one contiguous row
    for (int it = tid; it < kmax * C; it += kET) {
      const int k = 1 + it / C, cp = it % C;
      const int j = k < K - 1 ? k : K - 1;
      const float* e = edge_b + ((size_t)s * K + j) * cc + cp;
      const double* gn = g_b + (size_t)(s + k) * C;
      double m = -INFINITY;
      for (int c = 0; c < C; ++c) m = fmax(m, (double)e[(size_t)c * C] + gn[c]);
      double r = m;
      if (m > -INFINITY) {
        double sum = 0.0;
        for (int c = 0; c < C; ++c) sum += exp((double)e[(size_t)c * C] + gn[c] - m);
        r = m + log(sum);
      }
      item[(size_t)(k - 1) * C + cp] = r;
    }
    __syncthreads();
    for (int cp = tid; cp < C; cp += kET) {
      double m = -INFINITY;
      for (int k = 1; k <= kmax; ++k) m = fmax(m, item[(size_t)(k - 1) * C + cp]);
      double r = m;
      if (m > -INFINITY) {
        double sum = 0.0;
        for (int k = 1; k <= kmax; ++k) sum += exp(item[(size_t)(k - 1) * C + cp] - m);
        r = m + log(sum);
      }
      g_b[(size_t)s * C + cp] = r;
    }
    __syncthreads();
  }
}

// log-semiring gradient: one thread per edge element
__global__ void escan_grad_kernel(int B, int N, int K, int C, const float* edge,
                                  const int64_t* lengths, const double* beta,
                                  const double* gamma, const double* logz,
                                  const float* grad_output, float* grad_edge) {
  const size_t cc = (size_t)C * C;
  const size_t per_b = (size_t)(N - 1) * K * cc;
  const size_t total = (size_t)B * per_b;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const int b = (int)(i / per_b);
    size_t r = i % per_b;
    const int cp = (int)(r % C);
    r /= C;
    const int c = (int)(r % C);
    r /= C;
    const int j = (int)(r % K);
    const int s = (int)(r / K);
    const int L = es_len(lengths, b);
    const int k = K > 1 ? j : 1;  // the duration that reads index j
    float v = 0.f;
    if (L >= 1 && L <= N && (K == 1 || j >= 1) && s + k <= L - 1) {
      const double x = beta[((size_t)b * N + s) * C + cp] + (double)edge[i] +
                       gamma[((size_t)b * N + s + k) * C + c] - logz[b];
      v = (float)((double)grad_output[b] * exp(x));
    }
    grad_edge[i] = v;
  }
}

// max-semiring gradient: zero everything, then one thread per sequence walks
// the first-maximum path and marks its edges
__global__ void escan_zero_kernel(size_t n, float* out) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    out[i] = 0.f;
}

__global__ void escan_path_kernel(int B, int N, int K, int C, const int64_t* lengths,
                                  const double* beta, const int32_t* bp,
                                  const float* grad_output, float* grad_edge) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  const int L = es_len(lengths, b);
  if (L < 2 || L > N) return;  // length 1: no edge on the path
  const size_t cc = (size_t)C * C;
  // the first maximal final label
  const double* fin = beta + ((size_t)b * N + L - 1) * C;
  int c = 0;
  for (int q = 1; q < C; ++q)
    if (fin[q] > fin[c]) c = q;
  const float g = grad_output[b];
  int n = L - 1;
  while (n > 0) {
    const int32_t p = bp[((size_t)b * N + n) * C + c];
    const int k = p & 0xffff, cp = p >> 16;
    const int s = n - k;
    const int j = k < K - 1 ? k : K - 1;
    grad_edge[(((size_t)b * (N - 1) + s) * K + j) * cc + (size_t)c * C + cp] += g;
    n = s;
    c = cp;
  }
}

int es_grid(size_t n, int threads) {
  size_t g = (n + threads - 1) / threads;
  if (g > device_sm_count() * 32) g = device_sm_count() * 32;
  return g < 1 ? 1 : (int)g;
}

}  // namespace

bool escan_supported(int K, int C) {
  return K >= 1 && C >= 1 && C <= 4096 && es_smem(K, C) * 8 <= 200 * 1024;
}

cudaError_t launch_escan_forward(int B, int N, int K, int C, const float* edge,
                                 const int64_t* lengths, int semiring, float* partition,
                                 double* logz, double* beta_tab, int32_t* bp, cudaStream_t s) {
  if (B <= 0) return cudaSuccess;
  const size_t bytes = es_smem(K, C) * 8;
  auto go = [&](auto kern) -> cudaError_t {
    cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e != cudaSuccess) return e;
    kern<<<B, kET, bytes, s>>>(N, K, C, edge, lengths, partition, logz, beta_tab, bp);
    return cudaGetLastError();
  };
  return semiring == SEMICRF_LOG ? go(escan_fwd_kernel<0>) : go(escan_fwd_kernel<1>);
}

cudaError_t launch_escan_backward(int B, int N, int K, int C, const float* edge,
                                  const int64_t* lengths, int semiring, const double* beta,
                                  const double* logz, const int32_t* bp, const float* grad_output,
                                  float* grad_edge, double* gamma, cudaStream_t s) {
  if (B <= 0 || N < 2) return cudaSuccess;
  const size_t nedge = (size_t)B * (N - 1) * K * C * C;
  if (semiring == SEMICRF_LOG) {
    const size_t bytes = es_smem(K, C) * 8;
    cudaError_t e = cudaFuncSetAttribute(escan_out_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e != cudaSuccess) return e;
    escan_out_kernel<<<B, kET, bytes, s>>>(N, K, C, edge, lengths, gamma);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    escan_grad_kernel<<<es_grid(nedge, 256), 256, 0, s>>>(B, N, K, C, edge, lengths, beta, gamma,
                                                          logz, grad_output, grad_edge);
    return cudaGetLastError();
  }
  escan_zero_kernel<<<es_grid(nedge, 256), 256, 0, s>>>(nedge, grad_edge);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  escan_path_kernel<<<(B + 127) / 128, 128, 0, s>>>(B, N, K, C, lengths, beta, bp, grad_output,
                                                   grad_edge);
  return cudaGetLastError();
}

}  // namespace semicrf
