// viterbi.cu -- GPU backtrace over the compact backpointers of the max chain.
//
// Reference: SemiMarkovCRFHead._traceback_single / _compute_segment_score
// (nn.py:444-555).  The max-semiring chain (chain.cu, SEMI=1, BP=true)
// stores, per position t and label c,
//   bp_k[t,c] : the winning duration (smallest k on ties, nn.py:494)
//   bp_c[s,c] : argmax_c' (alpha[s,c'] + tr[c',c]) (first index, nn.py:491)
// and final_c = argmax_c alpha[L,c] (first index, nn.py:501).  The backtrace
// walks t = L -> 0 exactly like nn.py:507-530, scoring each segment with the
// float32 content, duration bias and transition summed in float64 (the
// reference sums the .item() values as Python floats).  Positions are below
// 2^15 and labels below 2^8 wherever the packed path is used (T <= 32767 is
// checked by the caller; C <= 32 there).

#include "semicrf_internal.cuh"

namespace semicrf {

__global__ void backtrace_kernel(int B, int T, int K, int C, const float* __restrict__ cum,
                                 const float* __restrict__ tr, const float* __restrict__ db,
                                 const int64_t* __restrict__ lengths, int64_t max_len,
                                 const int16_t* __restrict__ bp_k,
                                 const uint8_t* __restrict__ bp_c, const int* __restrict__ final_c,
                                 int32_t* seg_start, int32_t* seg_end, int32_t* seg_label,
                                 double* seg_score, int32_t* nseg) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  long long lr = lengths[b];
  const int L = lr < 0 ? 0 : (lr > T ? T : (int)lr);
  nseg[b] = 0;
  if (L == 0 || (int64_t)L > max_len) return;
  const size_t off = (size_t)b * T;
  const float* cum_b = cum + (size_t)b * (T + 1) * C;
  int t = L, c = final_c[b], n = 0;
  if (c < 0 || c >= C) c = 0;
  while (t > 0 && n < T) {
    const int k = bp_k[((size_t)b * (T + 1) + t) * C + c];
    if (k <= 0 || k > t) break;  // nn.py:511-513
    const int st = t - k, en = t - 1;
    int cp = bp_c[((size_t)b * (T + 1) + st) * C + c];
    if (cp >= C) cp = 0;
    const float content = cum_b[(size_t)(en + 1) * C + c] - cum_b[(size_t)st * C + c];
    const int dur = en - st + 1;
    const int di = dur < K - 1 ? dur : K - 1;
    seg_start[off + n] = st;
    seg_end[off + n] = en;
    seg_label[off + n] = c;
    seg_score[off + n] = (double)content + (double)db[(size_t)di * C + c] + (double)tr[cp * C + c];
    ++n;
    t = st;
    c = cp;
  }
  for (int i = 0; i < n / 2; ++i) {  // segments.reverse()
    const size_t x = off + i, y = off + n - 1 - i;
    int32_t v;
    v = seg_start[x]; seg_start[x] = seg_start[y]; seg_start[y] = v;
    v = seg_end[x]; seg_end[x] = seg_end[y]; seg_end[y] = v;
    v = seg_label[x]; seg_label[x] = seg_label[y]; seg_label[y] = v;
    const double d = seg_score[x]; seg_score[x] = seg_score[y]; seg_score[y] = d;
  }
  nseg[b] = n;
}

// Packed variant for the warp chain (vchain.cu): bp[t,c] = k | c_src << 8,
// where c_src is the source label at the segment start (the bp_c of the
// start).  One CTA per sequence stages the sequence's packed backpointers in
// shared memory; thread 0 walks them (one shared-memory load per segment)
// and records the path, then all threads write the segments in order.
constexpr int kBtThreads = 128;

__global__ void __launch_bounds__(kBtThreads) backtrace_packed_kernel(
    int B, int T, int K, int C, const float* __restrict__ cum, const float* __restrict__ tr,
    const float* __restrict__ db, const int64_t* __restrict__ lengths, int64_t max_len,
    const uint16_t* __restrict__ bp, const int* __restrict__ final_c, int32_t* seg_start,
    int32_t* seg_end, int32_t* seg_label, double* seg_score, int32_t* nseg) {
  extern __shared__ __align__(16) unsigned char btsm[];
  __shared__ int s_n;
  const int b = blockIdx.x;
  const long long lr = lengths[b];
  const int L = lr < 0 ? 0 : (lr > T ? T : (int)lr);
  if (L == 0 || (int64_t)L > max_len) {
    if (threadIdx.x == 0) nseg[b] = 0;
    return;
  }
  uint16_t* sbp = reinterpret_cast<uint16_t*>(btsm);  // [(L+1) * C]
  const size_t nbp = (size_t)(L + 1) * C;
  uint32_t* path = reinterpret_cast<uint32_t*>(btsm + ((2 * nbp + 15) & ~size_t(15)));  // [L]
  const uint16_t* bp_b = bp + (size_t)b * (T + 1) * C;
  for (size_t i = threadIdx.x; i < nbp; i += kBtThreads) sbp[i] = bp_b[i];
  __syncthreads();
  if (threadIdx.x == 0) {
    int t = L, c = final_c[b], n = 0;
    if (c < 0 || c >= C) c = 0;
    while (t > 0 && n < L) {
      const int p = sbp[(size_t)t * C + c];
      const int k = p & 255;
      if (k <= 0 || k > t) break;  // nn.py:511-513
      int cp = p >> 8;
      if (cp >= C) cp = 0;
      path[n++] = (uint32_t)t | ((uint32_t)c << 16) | ((uint32_t)cp << 24);
      t -= k;
      c = cp;
    }
    s_n = n;
    nseg[b] = n;
  }
  __syncthreads();
  const int n = s_n;
  const size_t off = (size_t)b * T;
  const float* cum_b = cum + (size_t)b * (T + 1) * C;
  for (int j = threadIdx.x; j < n; j += kBtThreads) {
    // path[n-1-j] is the j-th segment from the start
    const uint32_t e = path[n - 1 - j];
    const int t = (int)(e & 0xffff), c = (int)((e >> 16) & 0xff), cp = (int)(e >> 24);
    const int k = sbp[(size_t)t * C + c] & 255;
    const int st = t - k, en = t - 1;
    const float content = cum_b[(size_t)(en + 1) * C + c] - cum_b[(size_t)st * C + c];
    const int di = k < K - 1 ? k : K - 1;
    seg_start[off + j] = st;
    seg_end[off + j] = en;
    seg_label[off + j] = c;
    seg_score[off + j] = (double)content + (double)db[(size_t)di * C + c] + (double)tr[cp * C + c];
  }
}

size_t backtrace_packed_smem(int T, int C) {
  const size_t nbp = (size_t)(T + 1) * C;
  return ((2 * nbp + 15) & ~size_t(15)) + 4 * (size_t)T;
}

cudaError_t launch_backtrace_packed(int B, int T, int K, int C, const float* cum,
                                    const float* tr, const float* db, const int64_t* lengths,
                                    int64_t max_len, const uint16_t* bp, const int* final_c,
                                    int32_t* seg_start, int32_t* seg_end, int32_t* seg_label,
                                    double* seg_score, int32_t* nseg, cudaStream_t s) {
  const size_t smem = backtrace_packed_smem(T, C);
  cudaError_t e = cudaFuncSetAttribute(backtrace_packed_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  backtrace_packed_kernel<<<B, kBtThreads, smem, s>>>(B, T, K, C, cum, tr, db, lengths, max_len,
                                                      bp, final_c, seg_start, seg_end, seg_label,
                                                      seg_score, nseg);
  return cudaGetLastError();
}

cudaError_t launch_backtrace(int B, int T, int K, int C, const float* cum, const float* tr,
                             const float* db, const int64_t* lengths, int64_t max_len,
                             const int16_t* bp_k, const uint8_t* bp_c, const int* final_c,
                             int32_t* seg_start, int32_t* seg_end, int32_t* seg_label,
                             double* seg_score, int32_t* nseg, cudaStream_t s) {
  const int bs = 64;
  backtrace_kernel<<<(B + bs - 1) / bs, bs, 0, s>>>(B, T, K, C, cum, tr, db, lengths, max_len,
                                                    bp_k, bp_c, final_c, seg_start, seg_end,
                                                    seg_label, seg_score, nseg);
  return cudaGetLastError();
}

}  // namespace semicrf
