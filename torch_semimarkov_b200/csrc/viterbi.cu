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
// reference sums the .item() values as Python floats).

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
