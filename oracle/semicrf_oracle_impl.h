/*
 * Body of the CPU oracle, instantiated twice by semicrf_oracle.c: once with
 * REAL=double (the parity oracle) and once with REAL=float (the CPU baseline
 * that mirrors the reference's fp32 CPU path).
 *
 * TEST INFRASTRUCTURE ONLY.  This file restates, loop by loop, the reference
 * implementation in torch-semimarkov 0.2.0:
 *   src/torch_semimarkov/streaming/pytorch_reference.py   (forward, backward)
 *   src/torch_semimarkov/nn.py                            (Viterbi traceback)
 *   src/torch_semimarkov/helpers.py                       (gold scoring)
 * It is linked only by tests/, bench.py's CPU legs and __graft_entry__.smoke()
 * as a checker.  The product (torch_semimarkov_b200) never calls it.
 *
 * Every batch element is independent in the reference (all its ops are
 * batched elementwise / reductions over non-batch dims), so each function
 * below loops over b and restates the per-sequence semantics.
 */

#define CAT2(a, b) a##b
#define CAT(a, b) CAT2(a, b)
#define FN(name) CAT(name, SUFFIX)

/* torch.logsumexp over a contiguous run: max + log(sum(exp(x - max))).
 * All inputs in this path are finite (NEG_INF is -1e9, not -inf). */
static REAL FN(lse_)(const REAL* x, int64_t n, int64_t stride) {
    REAL m = x[0];
    for (int64_t i = 1; i < n; ++i) {
        if (x[i * stride] > m) m = x[i * stride];
    }
    if (isinf(m)) return m;
    REAL s = 0;
    for (int64_t i = 0; i < n; ++i) s += EXP(x[i * stride] - m);
    return m + LOG(s);
}

/* max with first-index tie break (torch.max on CPU). */
static REAL FN(max_)(const REAL* x, int64_t n, int64_t stride, int64_t* arg) {
    REAL m = x[0];
    int64_t a = 0;
    for (int64_t i = 1; i < n; ++i) {
        if (x[i * stride] > m) {
            m = x[i * stride];
            a = i;
        }
    }
    if (arg) *arg = a;
    return m;
}

/* compute_edge_block_streaming (pytorch_reference.py:48-113) for one batch
 * element: edge[c_dst*C + c_src] for a segment starting at `start` with
 * duration k.  tr is (C,C) src-major or (K,C,C) indexed by k. */
static void FN(edge_block_)(const REAL* cum_b, const REAL* tr, int tr_ndim, const REAL* db,
                            const REAL* ps_b, const REAL* pe_b, int64_t K, int64_t C,
                            int64_t start, int64_t k, REAL* edge) {
    int64_t dur_idx = k < K - 1 ? k : K - 1; /* :90-91 */
    const REAL* trk = tr_ndim == 2 ? tr : tr + k * C * C; /* :104-109 */
    for (int64_t cd = 0; cd < C; ++cd) {
        REAL seg = cum_b[(start + k) * C + cd] - cum_b[start * C + cd]; /* :87 */
        seg = seg + db[dur_idx * C + cd];                               /* :92 */
        if (ps_b) seg = seg + ps_b[start * C + cd];                     /* :95-96 */
        if (pe_b) seg = seg + pe_b[(start + k - 1) * C + cd];           /* :97-98 */
        for (int64_t cs = 0; cs < C; ++cs) edge[cd * C + cs] = seg + trk[cs * C + cd]; /* :111 */
    }
}

/* semi_crf_streaming_forward_pytorch (pytorch_reference.py:116-273).
 * partition: (B,), ring_ckpts: (B, N, K, C) with N = ceil(T/S) (:190). */
int FN(oracle_forward_)(const REAL* cum, const REAL* tr, int tr_ndim, const REAL* db,
                        const int64_t* lengths, const REAL* ps, const REAL* pe, int64_t B,
                        int64_t T, int64_t K, int64_t C, int semiring, int64_t S,
                        REAL* partition, REAL* ring_ckpts, int nthreads) {
    if (K < 1 || C < 1 || T < 0 || B < 0 || S < K) return 1;
    int64_t N = (T + S - 1) / S;
    int64_t b;
#pragma omp parallel for num_threads(nthreads > 0 ? nthreads : 1) schedule(dynamic, 1)
    for (b = 0; b < B; ++b) {
        const REAL* cum_b = cum + b * (T + 1) * C;
        const REAL* ps_b = ps ? ps + b * T * C : NULL;
        const REAL* pe_b = pe ? pe + b * T * C : NULL;
        int64_t L = lengths[b];
        REAL* ring = (REAL*)malloc(sizeof(REAL) * K * C);
        REAL* fin = (REAL*)malloc(sizeof(REAL) * C);
        REAL* edge = (REAL*)malloc(sizeof(REAL) * C * C);
        REAL* sc = (REAL*)malloc(sizeof(REAL) * C);
        int64_t kcap = K > 1 ? K - 1 : 1;
        REAL* over_src = (REAL*)malloc(sizeof(REAL) * kcap * C);
        REAL* alpha_t = (REAL*)malloc(sizeof(REAL) * C);
        REAL* ck = ring_ckpts ? ring_ckpts + b * N * K * C : NULL;
        for (int64_t i = 0; i < K * C; ++i) ring[i] = NEG_INF_R; /* :198 */
        for (int64_t c = 0; c < C; ++c) ring[c] = 0;             /* :199 */
        if (ck) {
            for (int64_t i = 0; i < N * K * C; ++i) ck[i] = NEG_INF_R; /* :193-195 */
            if (N > 0)
                for (int64_t i = 0; i < K * C; ++i) ck[i] = ring[i]; /* :202 */
        }
        for (int64_t c = 0; c < C; ++c) fin[c] = NEG_INF_R; /* :205 */
        for (int64_t t = 1; t <= T; ++t) {                   /* :208 */
            int active = t <= L;                             /* :210 */
            int64_t k_eff = (K - 1) < t ? (K - 1) : t;       /* :213 */
            int64_t nk = k_eff + 1 > 2 ? k_eff : 1;          /* range(1, max(k_eff+1, 2)) */
            for (int64_t k = 1; k <= nk; ++k) {
                int64_t start = t - k;
                const REAL* aprev = ring + (start % K) * C; /* :220-221 */
                FN(edge_block_)(cum_b, tr, tr_ndim, db, ps_b, pe_b, K, C, start, k, edge);
                for (int64_t cd = 0; cd < C; ++cd) {
                    for (int64_t cs = 0; cs < C; ++cs) sc[cs] = aprev[cs] + edge[cd * C + cs]; /* :229 */
                    over_src[(k - 1) * C + cd] =
                        semiring == 0 ? FN(lse_)(sc, C, 1) : FN(max_)(sc, C, 1, NULL); /* :235-241 */
                }
            }
            for (int64_t cd = 0; cd < C; ++cd)
                alpha_t[cd] = semiring == 0 ? FN(lse_)(over_src + cd, nk, C)
                                            : FN(max_)(over_src + cd, nk, C, NULL);
            if (active)
                for (int64_t c = 0; c < C; ++c) ring[(t % K) * C + c] = alpha_t[c]; /* :244-247 */
            if (ck && t % S == 0) {                                                  /* :250 */
                int64_t idx = t / S;
                if (idx < N && active)
                    for (int64_t i = 0; i < K * C; ++i) ck[idx * K * C + i] = ring[i]; /* :253-258 */
            }
            if (t == L)
                for (int64_t c = 0; c < C; ++c) fin[c] = alpha_t[c]; /* :263-265 */
        }
        partition[b] = semiring == 0 ? FN(lse_)(fin, C, 1) : FN(max_)(fin, C, 1, NULL); /* :268-271 */
        free(ring);
        free(fin);
        free(edge);
        free(sc);
        free(over_src);
        free(alpha_t);
    }
    return 0;
}

/* semi_crf_streaming_backward_pytorch (pytorch_reference.py:276-525).
 * Outputs are per batch element, exactly like the reference:
 *   grad_cum (B,T+1,C), grad_tr (B,C,C) or (B,K,C,C), grad_db (B,K,C),
 *   grad_ps/grad_pe (B,T,C) when the corresponding projection is given.
 * ring_ckpts has N checkpoints of shape (K,C); S is the forward's interval. */
int FN(oracle_backward_)(const REAL* cum, const REAL* tr, int tr_ndim, const REAL* db,
                         const int64_t* lengths, const REAL* ps, const REAL* pe, int64_t B,
                         int64_t T, int64_t K, int64_t C, int semiring, const REAL* logZ,
                         const REAL* ring_ckpts, int64_t N, int64_t S, REAL* grad_cum,
                         REAL* grad_tr, REAL* grad_db, REAL* grad_ps, REAL* grad_pe,
                         int nthreads) {
    if (K < 1 || C < 1 || T < 0 || B < 0) return 1;
    int64_t eff = S > K ? S : K; /* :341 */
    int64_t seg_size = eff + K;  /* :357 */
    int64_t trsz = tr_ndim == 2 ? C * C : K * C * C;
    int64_t b;
#pragma omp parallel for num_threads(nthreads > 0 ? nthreads : 1) schedule(dynamic, 1)
    for (b = 0; b < B; ++b) {
        const REAL* cum_b = cum + b * (T + 1) * C;
        const REAL* ps_b = ps ? ps + b * T * C : NULL;
        const REAL* pe_b = pe ? pe + b * T * C : NULL;
        REAL* gc = grad_cum + b * (T + 1) * C;
        REAL* gt = grad_tr + b * trsz;
        REAL* gd = grad_db + b * K * C;
        REAL* gps = (grad_ps && ps) ? grad_ps + b * T * C : NULL;
        REAL* gpe = (grad_pe && pe) ? grad_pe + b * T * C : NULL;
        int64_t L = lengths[b];
        REAL lz = logZ[b];
        for (int64_t i = 0; i < (T + 1) * C; ++i) gc[i] = 0;
        for (int64_t i = 0; i < trsz; ++i) gt[i] = 0;
        for (int64_t i = 0; i < K * C; ++i) gd[i] = 0;
        if (gps)
            for (int64_t i = 0; i < T * C; ++i) gps[i] = 0;
        if (gpe)
            for (int64_t i = 0; i < T * C; ++i) gpe[i] = 0;
        REAL* aseg = (REAL*)malloc(sizeof(REAL) * seg_size * C);
        REAL* bring = (REAL*)malloc(sizeof(REAL) * K * C);
        REAL* aring = (REAL*)malloc(sizeof(REAL) * K * C);
        REAL* edge = (REAL*)malloc(sizeof(REAL) * C * C);
        REAL* sc = (REAL*)malloc(sizeof(REAL) * C);
        int64_t kcap = K > 1 ? K - 1 : 1;
        int64_t kcap2 = (K - 1) > T ? (K - 1) : T; /* max_k = min(K-1, T-t) <= K-1 */
        if (kcap2 < 1) kcap2 = 1;
        REAL* over_src = (REAL*)malloc(sizeof(REAL) * kcap * C);
        REAL* alpha_t = (REAL*)malloc(sizeof(REAL) * C);
        REAL* msd = (REAL*)malloc(sizeof(REAL) * C);
        REAL* sfb = (REAL*)malloc(sizeof(REAL) * kcap * C * C);
        REAL* tmp = (REAL*)malloc(sizeof(REAL) * (kcap > C ? kcap : C) * C);
        for (int64_t i = 0; i < K * C; ++i) bring[i] = NEG_INF_R; /* :361 */
        for (int64_t c = 0; c < C; ++c) bring[(L % K) * C + c] = 0; /* :366-368 */
        for (int64_t ck = N - 1; ck >= 0; --ck) {                    /* :373 */
            int64_t seg_start = ck * S;                               /* :374 */
            int64_t seg_end = (ck + 1) * S < T ? (ck + 1) * S : T;    /* :375 */
            for (int64_t i = 0; i < seg_size * C; ++i) aseg[i] = NEG_INF_R; /* :378 */
            const REAL* ckp = ring_ckpts + (b * N + ck) * K * C;
            for (int64_t i = 0; i < K * C; ++i) aring[i] = ckp[i];                 /* :381 */
            for (int64_t c = 0; c < C; ++c) aseg[c] = aring[(seg_start % K) * C + c]; /* :384 */
            for (int64_t t = seg_start + 1; t < seg_end; ++t) {                    /* :387 */
                int active = t < L;                                                /* :388 */
                int64_t k_eff = (K - 1) < t ? (K - 1) : t;
                int64_t nk = k_eff + 1 > 2 ? k_eff : 1;
                for (int64_t k = 1; k <= nk; ++k) {
                    int64_t start = t - k;
                    const REAL* aprev = aring + (start % K) * C;
                    FN(edge_block_)(cum_b, tr, tr_ndim, db, ps_b, pe_b, K, C, start, k, edge);
                    for (int64_t cd = 0; cd < C; ++cd) {
                        for (int64_t cs = 0; cs < C; ++cs) sc[cs] = aprev[cs] + edge[cd * C + cs];
                        over_src[(k - 1) * C + cd] =
                            semiring == 0 ? FN(lse_)(sc, C, 1) : FN(max_)(sc, C, 1, NULL);
                    }
                }
                for (int64_t cd = 0; cd < C; ++cd)
                    alpha_t[cd] = semiring == 0 ? FN(lse_)(over_src + cd, nk, C)
                                                : FN(max_)(over_src + cd, nk, C, NULL);
                if (active) {
                    for (int64_t c = 0; c < C; ++c) aring[(t % K) * C + c] = alpha_t[c]; /* :415-417 */
                    for (int64_t c = 0; c < C; ++c) aseg[(t - seg_start) * C + c] = alpha_t[c]; /* :420-423 */
                }
            }
            for (int64_t t = seg_end - 1; t >= seg_start; --t) { /* :426 */
                const REAL* at = aseg + (t - seg_start) * C;
                if (!(t < L)) continue; /* :432-434 */
                int64_t max_k = (K - 1) < (T - t) ? (K - 1) : (T - t);
                int64_t nk = max_k + 1 > 2 ? max_k : 1; /* :440 */
                int64_t nvalid = 0;
                for (int64_t k = 1; k <= nk; ++k) {
                    int64_t end = t + k;
                    if (!(end <= L)) continue; /* :443-446 */
                    const REAL* bn = bring + (end % K) * C;
                    FN(edge_block_)(cum_b, tr, tr_ndim, db, ps_b, pe_b, K, C, t, k, edge);
                    for (int64_t cd = 0; cd < C; ++cd) {
                        REAL s = 0;
                        for (int64_t cs = 0; cs < C; ++cs) {
                            REAL lm = at[cs] + edge[cd * C + cs] + bn[cd] - lz; /* :458-463 */
                            REAL m = EXP(lm);                                    /* :464 */
                            s += m;
                            if (tr_ndim == 2)
                                gt[cs * C + cd] += m; /* :483 */
                            else
                                gt[k * C * C + cs * C + cd] += m; /* :485-487 */
                        }
                        msd[cd] = s;
                    }
                    int64_t dur_idx = k < K - 1 ? k : K - 1;
                    for (int64_t cd = 0; cd < C; ++cd) {
                        gc[end * C + cd] += msd[cd];    /* :475 */
                        gc[t * C + cd] -= msd[cd];      /* :477 */
                        gd[dur_idx * C + cd] += msd[cd]; /* :493 */
                        if (gps) gps[t * C + cd] += msd[cd];         /* :497 */
                        if (gpe) gpe[(end - 1) * C + cd] += msd[cd]; /* :499 */
                    }
                    for (int64_t cd = 0; cd < C; ++cd)
                        for (int64_t cs = 0; cs < C; ++cs)
                            sfb[(nvalid * C + cd) * C + cs] = edge[cd * C + cs] + bn[cd]; /* :502 */
                    ++nvalid;
                }
                if (nvalid > 0) { /* :511-523 */
                    for (int64_t v = 0; v < nvalid; ++v)
                        for (int64_t cs = 0; cs < C; ++cs)
                            tmp[v * C + cs] = semiring == 0
                                                  ? FN(lse_)(sfb + v * C * C + cs, C, C)
                                                  : FN(max_)(sfb + v * C * C + cs, C, C, NULL);
                    for (int64_t cs = 0; cs < C; ++cs)
                        bring[(t % K) * C + cs] = semiring == 0
                                                      ? FN(lse_)(tmp + cs, nvalid, C)
                                                      : FN(max_)(tmp + cs, nvalid, C, NULL);
                }
            }
        }
        free(aseg);
        free(bring);
        free(aring);
        free(edge);
        free(sc);
        free(over_src);
        free(alpha_t);
        free(msd);
        free(sfb);
        free(tmp);
    }
    return 0;
}

/* SemiMarkovCRFHead._traceback_single + _compute_segment_score
 * (nn.py:444-555) for every sequence with 0 < L <= max_len.
 * tr is (C,C).  Segments are written in order into seg_* at offset
 * b * T; nseg[b] = count (0 for skipped sequences).  score[b] is the max
 * of alpha[L] (the streaming max forward returns the same value). */
int FN(oracle_viterbi_)(const REAL* cum, const REAL* tr, const REAL* db, const int64_t* lengths,
                        int64_t B, int64_t T, int64_t K, int64_t C, int64_t max_len,
                        REAL* score, int64_t* seg_start, int64_t* seg_end, int64_t* seg_label,
                        double* seg_score, int64_t* nseg, int nthreads) {
    if (K < 1 || C < 1 || T < 0 || B < 0) return 1;
    int64_t b;
#pragma omp parallel for num_threads(nthreads > 0 ? nthreads : 1) schedule(dynamic, 1)
    for (b = 0; b < B; ++b) {
        const REAL* cum_b = cum + b * (T + 1) * C;
        int64_t L = lengths[b];
        nseg[b] = 0;
        if (L <= 0) {
            score[b] = NEG_INF_R;
            continue;
        }
        REAL* alpha = (REAL*)malloc(sizeof(REAL) * (L + 1) * C);
        int64_t* bpk = (int64_t*)calloc((L + 1) * C, sizeof(int64_t));
        int64_t* bpc = (int64_t*)calloc((L + 1) * C, sizeof(int64_t));
        REAL* edge = (REAL*)malloc(sizeof(REAL) * C * C);
        REAL* cand = (REAL*)malloc(sizeof(REAL) * C);
        for (int64_t i = 0; i < (L + 1) * C; ++i) alpha[i] = NEG_INF_R; /* :464 */
        for (int64_t c = 0; c < C; ++c) alpha[c] = 0;                   /* :465 */
        for (int64_t t = 1; t <= L; ++t) {                              /* :472 */
            int64_t k_eff = (K - 1) < t ? (K - 1) : t;
            int64_t nk = k_eff + 1 > 2 ? k_eff : 1;
            for (int64_t k = 1; k <= nk; ++k) {
                int64_t start = t - k;
                FN(edge_block_)(cum_b, tr, 2, db, NULL, NULL, K, C, start, k, edge);
                for (int64_t cd = 0; cd < C; ++cd) {
                    for (int64_t cs = 0; cs < C; ++cs)
                        cand[cs] = alpha[start * C + cs] + edge[cd * C + cs]; /* :488 */
                    int64_t arg;
                    REAL best = FN(max_)(cand, C, 1, &arg); /* :491 */
                    if (best > alpha[t * C + cd]) {         /* :494 */
                        alpha[t * C + cd] = best;
                        bpk[t * C + cd] = k;
                        bpc[t * C + cd] = arg;
                    }
                }
            }
        }
        int64_t bc;
        score[b] = FN(max_)(alpha + L * C, C, 1, &bc); /* :500-501 */
        int64_t t = L, c = bc, n = 0;
        int64_t* ss = seg_start + b * T;
        int64_t* se = seg_end + b * T;
        int64_t* sl = seg_label + b * T;
        double* sv = seg_score + b * T;
        if (L <= max_len) {
            while (t > 0) { /* :507 */
                int64_t k = bpk[t * C + c];
                int64_t cp = bpc[t * C + c];
                if (k == 0) break; /* :511-513 */
                int64_t st = t - k, en = t - 1;
                /* _compute_segment_score (nn.py:533-555): .item() values summed as
                 * Python floats. */
                REAL content = cum_b[(en + 1) * C + c] - cum_b[st * C + c];
                int64_t dur = en - st + 1;
                int64_t di = dur < K - 1 ? dur : K - 1;
                ss[n] = st;
                se[n] = en;
                sl[n] = c;
                sv[n] = (double)content + (double)db[di * C + c] + (double)tr[cp * C + c];
                ++n;
                t = st;
                c = cp;
            }
            for (int64_t i = 0; i < n / 2; ++i) { /* segments.reverse() */
                int64_t j = n - 1 - i, x;
                double y;
                x = ss[i]; ss[i] = ss[j]; ss[j] = x;
                x = se[i]; se[i] = se[j]; se[j] = x;
                x = sl[i]; sl[i] = sl[j]; sl[j] = x;
                y = sv[i]; sv[i] = sv[j]; sv[j] = y;
            }
            nseg[b] = n;
        }
        free(alpha);
        free(bpk);
        free(bpc);
        free(edge);
        free(cand);
    }
    return 0;
}

/* score_gold_vectorized (helpers.py:365-544): gold segmentation score per
 * sequence.  Returns 2 if T == 1 and K < 2 (the reference indexes
 * duration_bias[1] there and raises). */
int FN(oracle_score_gold_)(const REAL* cum, const int64_t* labels, const int64_t* lengths,
                           const REAL* tr, const REAL* db, int64_t B, int64_t T, int64_t K,
                           int64_t C, REAL* out) {
    if (T == 0) { /* :402-403 */
        for (int64_t b = 0; b < B; ++b) out[b] = 0;
        return 0;
    }
    if (T == 1) { /* :406-415 */
        if (K < 2) return 2;
        for (int64_t b = 0; b < B; ++b) {
            int64_t l0 = labels[b];
            REAL content = cum[(b * 2 + 1) * C + l0] - cum[(b * 2) * C + l0];
            REAL s = content + db[1 * C + l0];
            out[b] = s * (REAL)(lengths[b] > 0);
        }
        return 0;
    }
    for (int64_t b = 0; b < B; ++b) {
        const REAL* cum_b = cum + b * (T + 1) * C;
        const int64_t* lab = labels + b * T;
        int64_t L = lengths[b];
        REAL total = 0;
        if (L <= 0) {
            out[b] = 0;
            continue;
        }
        int64_t st = 0, prev = -1;
        for (int64_t p = 0; p < L; ++p) {
            int is_end = (p == L - 1) || (lab[p] != lab[p + 1]); /* :423-429, :460-466 */
            if (!is_end) continue;
            int64_t c = lab[st];
            REAL content = cum_b[(p + 1) * C + c] - cum_b[st * C + c]; /* :496-508 */
            int64_t dur = p - st + 1;
            int64_t di = dur < 1 ? 1 : dur;                       /* clamp(1, K-1) :511-514 */
            if (di > K - 1) di = K - 1;
            REAL dterm = db[di * C + c];
            REAL trans = prev >= 0 ? tr[prev * C + c] : 0;        /* :525-536 */
            total += content + dterm + trans;                      /* :539-543 */
            prev = c;
            st = p + 1;
        }
        out[b] = total;
    }
    return 0;
}

#undef FN
#undef CAT
#undef CAT2
