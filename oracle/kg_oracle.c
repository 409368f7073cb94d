/*
 * TEST INFRASTRUCTURE ONLY -- CPU restatement of the reference kernels (see kg_oracle.h).
 * Built with -ffp-contract=off so every multiply and add rounds separately, as the
 * reference's npu_demo helpers do when g++ compiles them for x86-64.
 */
#include "kg_oracle.h"

#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static float bf16_to_f32(uint16_t h) {
    uint32_t u = ((uint32_t)h) << 16;
    float f;
    memcpy(&f, &u, sizeof(f));
    return f;
}

static float load_value(const void* base, int dtype, long long index) {
    if (dtype == KGO_BF16) {
        return bf16_to_f32(((const uint16_t*)base)[index]);
    }
    return ((const float*)base)[index];
}

static long long min_ll(long long a, long long b) { return a < b ? a : b; }
static long long max_ll(long long a, long long b) { return a > b ? a : b; }

/* npu_demo::matmul, include/npu_demo/Kernel.h:928-946: acc_value starts at 0 (or the old
 * out value when acc != 0) and adds lhs*rhs in k order, rounding to float each step. */
int kgo_tile_matmul(float* out, const float* lhs, const float* rhs, long long m, long long k, long long n, int acc) {
    if (!out || !lhs || !rhs || m <= 0 || k <= 0 || n <= 0) {
        return 1;
    }
    for (long long mi = 0; mi < m; ++mi) {
        for (long long ni = 0; ni < n; ++ni) {
            float acc_value = acc ? out[mi * n + ni] : 0.0f;
            for (long long ki = 0; ki < k; ++ki) {
                float prod = lhs[mi * k + ki] * rhs[ki * n + ni];
                acc_value = acc_value + prod;
            }
            out[mi * n + ni] = acc_value;
        }
    }
    return 0;
}

/* kernel/matmul/inputs_dynamic_tile_dynamic.py:84-113. For each (h0, w0) output tile the
 * accumulator starts at zero; every k tile produces `partial = lhs_tile . rhs_tile`
 * (npu_demo::matmul) which is added into the accumulator (kernel.add); after the k loop
 * the optional rank-1 bias is broadcast-added and the tile is written out. Rows are
 * independent, so a row range reproduces exactly the rows of a full run. */
int kgo_matmul(float* out, const void* lhs, const void* rhs, int in_dtype, const float* bias,
               long long H, long long K, long long W,
               long long tile_h, long long tile_w, long long tile_k,
               long long row_begin, long long row_end) {
    if (!out || !lhs || !rhs || H <= 0 || K <= 0 || W <= 0 || tile_h <= 0 || tile_w <= 0 || tile_k <= 0) {
        return 1;
    }
    if (in_dtype != KGO_F32 && in_dtype != KGO_BF16) {
        return 1;
    }
    row_begin = max_ll(row_begin, 0);
    row_end = min_ll(row_end, H);
    if (row_begin >= row_end) {
        return 0;
    }
    float* acc = (float*)malloc(sizeof(float) * (size_t)tile_w);
    float* lhs_row = (float*)malloc(sizeof(float) * (size_t)tile_k);
    float* rhs_tile = (float*)malloc(sizeof(float) * (size_t)(tile_k * tile_w));
    if (!acc || !lhs_row || !rhs_tile) {
        free(acc);
        free(lhs_row);
        free(rhs_tile);
        return 2;
    }
    for (long long h0 = 0; h0 < H; h0 += tile_h) {
        const long long cur_h = min_ll(tile_h, H - h0);
        const long long r0 = max_ll(h0, row_begin);
        const long long r1 = min_ll(h0 + cur_h, row_end);
        if (r0 >= r1) {
            continue;
        }
        for (long long w0 = 0; w0 < W; w0 += tile_w) {
            const long long cur_w = min_ll(tile_w, W - w0);
            for (long long row = r0; row < r1; ++row) {
                for (long long j = 0; j < cur_w; ++j) {
                    acc[j] = 0.0f; /* fill(acc, 0) */
                }
                for (long long k0 = 0; k0 < K; k0 += tile_k) {
                    const long long cur_k = min_ll(tile_k, K - k0);
                    for (long long kk = 0; kk < cur_k; ++kk) {
                        lhs_row[kk] = load_value(lhs, in_dtype, row * K + k0 + kk);
                        for (long long j = 0; j < cur_w; ++j) {
                            rhs_tile[kk * cur_w + j] = load_value(rhs, in_dtype, (k0 + kk) * W + w0 + j);
                        }
                    }
                    for (long long j = 0; j < cur_w; ++j) {
                        float partial = 0.0f;
                        for (long long kk = 0; kk < cur_k; ++kk) {
                            float prod = lhs_row[kk] * rhs_tile[kk * cur_w + j];
                            partial = partial + prod;
                        }
                        acc[j] = acc[j] + partial; /* kernel.add(acc, acc, partial) */
                    }
                }
                for (long long j = 0; j < cur_w; ++j) {
                    float value = acc[j];
                    if (bias) {
                        value = value + bias[w0 + j];
                    }
                    out[row * W + w0 + j] = value;
                }
            }
        }
    }
    free(acc);
    free(lhs_row);
    free(rhs_tile);
    return 0;
}

/* kernel/conv2d/inputs_dynamic_tile_dynamic.py:142-205. Per (f0, n0, ho0, wo0, ni) tile the
 * accumulator starts at zero; per input-channel tile c0 the window is unrolled by img2col2d
 * into col[cur_c*KH*KW, cur_ho*cur_wo] (zero outside the input), `out2 = weight2 . col2`
 * is computed by npu_demo::matmul in (c, kh, kw) order and added into the accumulator;
 * then the optional bias is added and the tile is written out. */
int kgo_conv2d(float* out, const void* input, const void* weight, int in_dtype, const float* bias,
               long long B, long long C, long long XH, long long XW,
               long long F, long long KH, long long KW,
               long long sh, long long sw, long long dh, long long dw,
               long long pt, long long pb, long long pl, long long pr,
               long long tile_f, long long tile_c, long long tile_n, long long tile_ho, long long tile_wo) {
    if (!out || !input || !weight || B <= 0 || C <= 0 || XH <= 0 || XW <= 0 || F <= 0 || KH <= 0 || KW <= 0) {
        return 1;
    }
    if (sh <= 0 || sw <= 0 || dh <= 0 || dw <= 0 || pt < 0 || pb < 0 || pl < 0 || pr < 0) {
        return 1;
    }
    if (tile_f <= 0 || tile_c <= 0 || tile_n <= 0 || tile_ho <= 0 || tile_wo <= 0) {
        return 1;
    }
    if (in_dtype != KGO_F32 && in_dtype != KGO_BF16) {
        return 1;
    }
    const long long HO = ((XH + pt + pb - dh * (KH - 1) - 1) / sh) + 1;
    const long long WO = ((XW + pl + pr - dw * (KW - 1) - 1) / sw) + 1;
    if (HO <= 0 || WO <= 0) {
        return 1;
    }
    const long long kmax = tile_c * KH * KW;
    const long long spatial_max = tile_ho * tile_wo;
    float* acc = (float*)malloc(sizeof(float) * (size_t)(tile_f * spatial_max));
    float* col = (float*)malloc(sizeof(float) * (size_t)(kmax * spatial_max));
    float* wt = (float*)malloc(sizeof(float) * (size_t)(tile_f * kmax));
    if (!acc || !col || !wt) {
        free(acc);
        free(col);
        free(wt);
        return 2;
    }
    for (long long f0 = 0; f0 < F; f0 += tile_f) {
        for (long long n0 = 0; n0 < B; n0 += tile_n) {
            for (long long ho0 = 0; ho0 < HO; ho0 += tile_ho) {
                for (long long wo0 = 0; wo0 < WO; wo0 += tile_wo) {
                    const long long cur_f = min_ll(tile_f, F - f0);
                    const long long cur_n = min_ll(tile_n, B - n0);
                    const long long cur_ho = min_ll(tile_ho, HO - ho0);
                    const long long cur_wo = min_ll(tile_wo, WO - wo0);
                    const long long spatial = cur_ho * cur_wo;
                    for (long long ni = 0; ni < cur_n; ++ni) {
                        const long long b = n0 + ni;
                        for (long long i = 0; i < cur_f * spatial; ++i) {
                            acc[i] = 0.0f;
                        }
                        for (long long c0 = 0; c0 < C; c0 += tile_c) {
                            const long long cur_c = min_ll(tile_c, C - c0);
                            const long long k_tile = cur_c * KH * KW;
                            /* img2col2d: col[(c,kh,kw), (ho,wo)] */
                            for (long long c = 0; c < cur_c; ++c) {
                                for (long long khi = 0; khi < KH; ++khi) {
                                    for (long long kwi = 0; kwi < KW; ++kwi) {
                                        const long long krow = (c * KH + khi) * KW + kwi;
                                        for (long long ho = 0; ho < cur_ho; ++ho) {
                                            const long long h = (ho0 + ho) * sh - pt + khi * dh;
                                            for (long long wo = 0; wo < cur_wo; ++wo) {
                                                const long long w = (wo0 + wo) * sw - pl + kwi * dw;
                                                float value = 0.0f;
                                                if (h >= 0 && h < XH && w >= 0 && w < XW) {
                                                    value = load_value(input, in_dtype, ((b * C + c0 + c) * XH + h) * XW + w);
                                                }
                                                col[krow * spatial + ho * cur_wo + wo] = value;
                                            }
                                        }
                                    }
                                }
                            }
                            for (long long f = 0; f < cur_f; ++f) {
                                for (long long kk = 0; kk < k_tile; ++kk) {
                                    const long long c = kk / (KH * KW);
                                    const long long rem = kk % (KH * KW);
                                    wt[f * k_tile + kk] = load_value(weight, in_dtype, ((f0 + f) * C + c0 + c) * KH * KW + rem);
                                }
                            }
                            /* out2 = weight2 . col2 (npu_demo::matmul), then acc += partial */
                            for (long long f = 0; f < cur_f; ++f) {
                                for (long long s = 0; s < spatial; ++s) {
                                    float partial = 0.0f;
                                    for (long long kk = 0; kk < k_tile; ++kk) {
                                        float prod = wt[f * k_tile + kk] * col[kk * spatial + s];
                                        partial = partial + prod;
                                    }
                                    acc[f * spatial + s] = acc[f * spatial + s] + partial;
                                }
                            }
                        }
                        for (long long f = 0; f < cur_f; ++f) {
                            for (long long ho = 0; ho < cur_ho; ++ho) {
                                for (long long wo = 0; wo < cur_wo; ++wo) {
                                    float value = acc[f * spatial + ho * cur_wo + wo];
                                    if (bias) {
                                        value = value + bias[f0 + f];
                                    }
                                    out[((b * F + f0 + f) * HO + ho0 + ho) * WO + wo0 + wo] = value;
                                }
                            }
                        }
                    }
                }
            }
        }
    }
    free(acc);
    free(col);
    free(wt);
    return 0;
}

/* kernel/flash_attention/inputs_dynamic_tile_dynamic.py:117-195, one query row at a time
 * (rows of a query tile are independent; padded tail rows are never written, line 193).
 * Per key tile: score = q . k^T (npu_demo::matmul), [extension: * scale], tail and
 * [extension: causal] entries are -inf; tile_max = reduce_max; m_next = max(m, tile_max);
 * p = exp(score - m_next); tile_sum = reduce_sum(p); old_scale = exp(m - m_next);
 * l = l * old_scale + tile_sum; o = o * old_scale + p . v. Output = o / l (double divide). */
int kgo_flash_attention(float* out, const void* q, const void* k, const void* v, int in_dtype,
                        long long B, long long H, long long S, long long D,
                        long long br, long long bc, float scale, int causal,
                        long long bh_begin, long long bh_end, long long q_begin, long long q_end) {
    if (!out || !q || !k || !v || B <= 0 || H <= 0 || S <= 0 || D <= 0 || br <= 0 || bc <= 0) {
        return 1;
    }
    if (in_dtype != KGO_F32 && in_dtype != KGO_BF16) {
        return 1;
    }
    bh_begin = max_ll(bh_begin, 0);
    bh_end = min_ll(bh_end, B * H);
    q_begin = max_ll(q_begin, 0);
    q_end = min_ll(q_end, S);
    float* qrow = (float*)malloc(sizeof(float) * (size_t)D);
    float* ktile = (float*)malloc(sizeof(float) * (size_t)(bc * D));
    float* vtile = (float*)malloc(sizeof(float) * (size_t)(bc * D));
    float* score = (float*)malloc(sizeof(float) * (size_t)bc);
    float* weighted = (float*)malloc(sizeof(float) * (size_t)D);
    if (!qrow || !ktile || !vtile || !score || !weighted) {
        free(qrow);
        free(ktile);
        free(vtile);
        free(score);
        free(weighted);
        return 2;
    }
    for (long long bh = bh_begin; bh < bh_end; ++bh) {
        const long long base = bh * S * D;
        for (long long row = q_begin; row < q_end; ++row) {
            for (long long d = 0; d < D; ++d) {
                qrow[d] = load_value(q, in_dtype, base + row * D + d);
                weighted[d] = 0.0f;
            }
            float m_state = -INFINITY;
            float sum_state = 0.0f;
            for (long long n0 = 0; n0 < S; n0 += bc) {
                const long long cur_bc = min_ll(bc, S - n0);
                for (long long j = 0; j < cur_bc; ++j) {
                    for (long long d = 0; d < D; ++d) {
                        ktile[j * D + d] = load_value(k, in_dtype, base + (n0 + j) * D + d);
                        vtile[j * D + d] = load_value(v, in_dtype, base + (n0 + j) * D + d);
                    }
                }
                /* Tail columns j >= cur_bc hold -inf (fill(score_tile, "-inf")); they can never
                 * raise the row maximum, so the reduction runs over the valid columns only. */
                float tile_max = -INFINITY;
                for (long long j = 0; j < cur_bc; ++j) {
                    float s = -INFINITY;
                    if (!(causal && n0 + j > row)) {
                        float dot = 0.0f;
                        for (long long d = 0; d < D; ++d) {
                            float prod = qrow[d] * ktile[j * D + d];
                            dot = dot + prod;
                        }
                        s = dot * scale;
                    }
                    score[j] = s;
                    /* reduce_max: first element, then value > current ? value : current */
                    tile_max = (j == 0) ? s : (s > tile_max ? s : tile_max);
                }
                const float m_next = m_state > tile_max ? m_state : tile_max;
                float tile_sum = 0.0f;
                for (long long j = 0; j < cur_bc; ++j) {
                    const float shifted = score[j] - m_next;
                    const float p = (float)exp((double)shifted);
                    score[j] = p;
                    tile_sum = tile_sum + p; /* tail columns contribute exp(-inf) = 0 */
                }
                const float old_shift = m_state - m_next;
                const float old_scale = (float)exp((double)old_shift);
                const float scaled_sum = sum_state * old_scale;
                sum_state = scaled_sum + tile_sum;
                for (long long d = 0; d < D; ++d) {
                    float partial = 0.0f;
                    for (long long j = 0; j < cur_bc; ++j) {
                        float prod = score[j] * vtile[j * D + d];
                        partial = partial + prod;
                    }
                    const float scaled = weighted[d] * old_scale;
                    weighted[d] = scaled + partial;
                }
                m_state = m_next;
            }
            for (long long d = 0; d < D; ++d) {
                out[base + row * D + d] = (float)((double)weighted[d] / (double)sum_state);
            }
        }
    }
    free(qrow);
    free(ktile);
    free(vtile);
    free(score);
    free(weighted);
    return 0;
}
