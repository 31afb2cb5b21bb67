// gold.cu -- score of the gold segmentation and its gradient.
//
// Reference: score_gold_vectorized (helpers.py:365-544).  Segments are the
// maximal runs of equal labels inside [0, length); a segment [st, en] with
// label c scores
//     cum[en+1,c] - cum[st,c] + db[clamp(en-st+1, 1, K-1), c] + tr[prev,c]
// (no transition for the first segment).  T == 1 uses db[1] directly
// (:406-415).  One thread walks one sequence; float64 accumulation.

#include "semicrf_internal.cuh"

namespace semicrf {

__device__ __forceinline__ int dur_index(int dur, int K) {
  int di = dur < 1 ? 1 : dur;  // clamp(1, K-1); torch.clamp with min > max gives max
  if (di > K - 1) di = K - 1;
  return di;
}

__global__ void gold_kernel(int B, int T, int K, int C, const float* __restrict__ cum,
                            const int64_t* __restrict__ labels,
                            const int64_t* __restrict__ lengths, const float* __restrict__ tr,
                            const float* __restrict__ db, float* __restrict__ out) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  long long lr = lengths[b];
  const int L = lr < 0 ? 0 : (lr > T ? T : (int)lr);
  const float* cb = cum + (size_t)b * (T + 1) * C;
  const int64_t* lab = labels + (size_t)b * T;
  if (T == 0) {
    out[b] = 0.f;
    return;
  }
  if (T == 1) {
    const int l0 = (int)lab[0];
    if (l0 < 0 || l0 >= C) {  // invalid label: reported as NaN, never read out of bounds
      out[b] = __int_as_float(0x7fc00000);
      return;
    }
    const float content = cb[1 * C + l0] - cb[l0];
    const float s = content + db[1 * C + l0];
    out[b] = L > 0 ? s : 0.f * s;
    return;
  }
  double total = 0.0;
  int st = 0, prev = -1;
  for (int p = 0; p < L; ++p) {
    if (!(p == L - 1 || lab[p] != lab[p + 1])) continue;
    const int c = (int)lab[st];
    if (c < 0 || c >= C) {
      out[b] = __int_as_float(0x7fc00000);
      return;
    }
    const float content = cb[(size_t)(p + 1) * C + c] - cb[(size_t)st * C + c];
    const float dterm = db[(size_t)dur_index(p - st + 1, K) * C + c];
    const float trans = prev >= 0 ? tr[prev * C + c] : 0.f;
    total += (double)((content + dterm) + trans);
    prev = c;
    st = p + 1;
  }
  out[b] = (float)total;
}

// grad_cum (B,T+1,C) must be zeroed by the caller's launch sequence; part is
// (B, C*C + K*C) per-sequence counts weighted by grad_out[b].
__global__ void gold_bwd_kernel(int B, int T, int K, int C, const int64_t* __restrict__ labels,
                                const int64_t* __restrict__ lengths,
                                const float* __restrict__ g, float* __restrict__ grad_cum,
                                float* __restrict__ part) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  long long lr = lengths[b];
  const int L = lr < 0 ? 0 : (lr > T ? T : (int)lr);
  float* gc = grad_cum + (size_t)b * (T + 1) * C;
  float* pt = part + (size_t)b * (C * C + K * C);
  float* pd = pt + C * C;
  const int64_t* lab = labels + (size_t)b * T;
  const float gb = g[b];
  if (T == 0) return;
  if (T == 1) {
    if (L > 0) {
      const int l0 = (int)lab[0];
      if (l0 < 0 || l0 >= C) return;
      gc[1 * C + l0] += gb;
      gc[l0] -= gb;
      pd[1 * C + l0] += gb;
    }
    return;
  }
  int st = 0, prev = -1;
  for (int p = 0; p < L; ++p) {
    if (!(p == L - 1 || lab[p] != lab[p + 1])) continue;
    const int c = (int)lab[st];
    if (c < 0 || c >= C) return;
    gc[(size_t)(p + 1) * C + c] += gb;
    gc[(size_t)st * C + c] -= gb;
    pd[(size_t)dur_index(p - st + 1, K) * C + c] += gb;
    if (prev >= 0) pt[prev * C + c] += gb;
    prev = c;
    st = p + 1;
  }
}

__global__ void zero_kernel(float* p, size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    p[i] = 0.f;
}

__global__ void sum_rows_kernel(int B, int n, const float* __restrict__ part, int stride,
                                float* __restrict__ out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  double acc = 0.0;
  for (int b = 0; b < B; ++b) acc += (double)part[(size_t)b * stride + i];
  out[i] = (float)acc;
}

cudaError_t launch_gold(int B, int T, int K, int C, const float* cum, const int64_t* labels,
                        const int64_t* lengths, const float* tr, const float* db, float* out,
                        cudaStream_t s) {
  gold_kernel<<<(B + 127) / 128, 128, 0, s>>>(B, T, K, C, cum, labels, lengths, tr, db, out);
  return cudaGetLastError();
}

cudaError_t launch_gold_backward(int B, int T, int K, int C, const int64_t* labels,
                                 const int64_t* lengths, const float* grad_out, float* grad_cum,
                                 float* grad_tr, float* grad_db, float* part, cudaStream_t s) {
  const size_t ngc = (size_t)B * (T + 1) * C;
  const size_t npart = (size_t)B * (C * C + K * C);
  zero_kernel<<<1184, 256, 0, s>>>(grad_cum, ngc);
  zero_kernel<<<1184, 256, 0, s>>>(part, npart);
  gold_bwd_kernel<<<(B + 127) / 128, 128, 0, s>>>(B, T, K, C, labels, lengths, grad_out,
                                                   grad_cum, part);
  const int stride = C * C + K * C;
  sum_rows_kernel<<<(C * C + 255) / 256, 256, 0, s>>>(B, C * C, part, stride, grad_tr);
  sum_rows_kernel<<<(K * C + 255) / 256, 256, 0, s>>>(B, K * C, part + C * C, stride, grad_db);
  return cudaGetLastError();
}

}  // namespace semicrf
