/* TEST INFRASTRUCTURE ONLY (see oracle.h): scalar restatement of the
 * int16 fixed-point GPT-2 forward primitives at the seam, one function per
 * reference kernel (cuda/volta_cuda_backend.cu:1442-1740; the CPU semantics
 * they freeze are rust/volta-gpt2/src/layer.rs and scripts/gpt2_fixed.py).
 * Every output, accumulator and the sticky error word follow the kernels'
 * definitions element by element. */
#include <stdint.h>
#include <stddef.h>

#include "oracle.h"

/* backend.cu:1442-1446 (floor division for negative numerators) */
static int64_t floor_div(int64_t a, int64_t b) {
    const int64_t q = a / b, r = a % b;
    return r < 0 ? q - 1 : q;
}

/* backend.cu:1448-1457: round half up, chained through 2^16 for shift > 16 */
static int64_t requant_rounded(int64_t acc, uint32_t shift) {
    int64_t stage = acc;
    uint32_t fin = shift;
    if (shift > 16) {
        const uint32_t first = shift - 16;
        stage = (stage + ((int64_t)1 << (first - 1))) >> first;
        fin = 16;
    }
    return (stage + ((int64_t)1 << (fin - 1))) >> fin;
}

/* backend.cu:1459-1465 */
static int16_t requant_no_clamp(int64_t acc, uint32_t shift, uint32_t* err) {
    const int64_t r = requant_rounded(acc, shift);
    if (r < INT16_MIN || r > INT16_MAX) *err = 1;
    return (int16_t)r;
}

/* backend.cu:1467-1476 */
static int16_t score_clamp17(int64_t acc, uint32_t shift, uint32_t* err) {
    const int64_t r = requant_rounded(acc, shift);
    if (r < -((int64_t)1 << 16) || r >= ((int64_t)1 << 16)) *err = 1;
    return (int16_t)(r < INT16_MIN ? INT16_MIN : (r > INT16_MAX ? INT16_MAX : r));
}

/* backend.cu:1482-1508 */
void or_fixed_embed(const uint32_t* tokens, const int16_t* wte, const int16_t* wpe, int64_t* acc_out,
                    int16_t* out, uint32_t* err, size_t rows, size_t d, size_t vocab, size_t positions,
                    size_t pos0, int32_t shift) {
    for (size_t row = 0; row < rows; ++row)
        for (size_t col = 0; col < d; ++col) {
            const size_t z = row * d + col;
            const uint32_t tok = tokens[row];
            if (tok >= vocab || pos0 + row >= positions) {
                *err = 1;
                acc_out[z] = 0;
                out[z] = 0;
                continue;
            }
            const int64_t acc = (int64_t)wte[(size_t)tok * d + col] + (int64_t)wpe[(pos0 + row) * d + col];
            acc_out[z] = acc;
            if (shift > 0) {
                out[z] = requant_no_clamp(acc, (uint32_t)shift, err);
            } else {
                const int64_t v = acc << (uint32_t)(-shift);
                if (v < INT16_MIN || v > INT16_MAX) *err = 1;
                out[z] = (int16_t)v;
            }
        }
}

/* backend.cu:1510-1549 */
void or_fixed_layer_norm(const int16_t* input, const int16_t* gain, const int16_t* bias, const int16_t* lut,
                         int64_t* means, int64_t* vars, int64_t* rin, int16_t* rout, int64_t* accs, int16_t* outs,
                         uint32_t* err, size_t rows, size_t d, uint32_t var_shift, uint32_t norm_shift) {
    for (size_t r = 0; r < rows; ++r) {
        const int16_t* row = input + r * d;
        int64_t sum = 0;
        for (size_t j = 0; j < d; ++j) sum += row[j];
        const int64_t di = (int64_t)d;
        const int64_t mean = floor_div(sum + di / 2, di);
        int64_t vs = 0;
        for (size_t j = 0; j < d; ++j) {
            const int64_t dl = (int64_t)row[j] - mean;
            vs += dl * dl;
        }
        const int64_t var = floor_div(vs + di / 2, di);
        int64_t ri = var >> var_shift;
        if (ri < 0 || ri >= ((int64_t)1 << 16)) {
            *err = 1;
            ri = 0;
        }
        const int16_t ro = lut[ri];
        means[r] = mean;
        vars[r] = var;
        rin[r] = ri;
        rout[r] = ro;
        for (size_t j = 0; j < d; ++j) {
            const int64_t dl = (int64_t)row[j] - mean;
            const int64_t acc = dl * (int64_t)ro * (int64_t)gain[j] + ((int64_t)bias[j] << norm_shift);
            accs[r * d + j] = acc;
            outs[r * d + j] = requant_no_clamp(acc, norm_shift, err);
        }
    }
}

/* backend.cu:1551-1574 (bias and residual optional: NULL) */
void or_fixed_gemm(const int16_t* input, const int16_t* w, const int16_t* bias, const int16_t* residual,
                   int64_t* accs, int16_t* req, int16_t* res_out, uint32_t* err, size_t m, size_t k, size_t n,
                   uint32_t shift) {
#pragma omp parallel for schedule(static)
    for (size_t i = 0; i < m; ++i) {
        uint32_t e = 0;
        for (size_t j = 0; j < n; ++j) {
            int64_t acc = 0;
            for (size_t q = 0; q < k; ++q) acc += (int64_t)input[i * k + q] * (int64_t)w[q * n + j];
            if (bias) acc += (int64_t)bias[j] << shift;
            const size_t z = i * n + j;
            accs[z] = acc;
            const int16_t qv = requant_no_clamp(acc, shift, &e);
            req[z] = qv;
            if (res_out) {
                const int32_t v = (int32_t)qv + residual[z];
                if (v < INT16_MIN || v > INT16_MAX) e = 1;
                res_out[z] = (int16_t)v;
            }
        }
        if (e) {
#pragma omp atomic write
            *err = 1;
        }
    }
}

/* backend.cu:1576-1587 */
void or_fixed_qkv_split(const int16_t* qkv, int16_t* q, int16_t* k, int16_t* v, size_t rows, size_t d) {
    for (size_t row = 0; row < rows; ++row)
        for (size_t col = 0; col < d; ++col) {
            const int16_t* src = qkv + row * 3 * d;
            q[row * d + col] = src[col];
            k[row * d + col] = src[d + col];
            v[row * d + col] = src[2 * d + col];
        }
}

static size_t packed_prefix(size_t row, size_t pos0) { return row * pos0 + row * (row + 1) / 2; }

/* backend.cu:1593-1617: causal-packed scores, head-major */
void or_fixed_attention_scores(const int16_t* q, const int16_t* k, int64_t* accs, int16_t* outs, uint32_t* err,
                               size_t rows, size_t seq, size_t pos0, size_t heads, size_t head_dim,
                               uint32_t shift) {
    const size_t d = heads * head_dim;
    const size_t per_head = rows * pos0 + rows * (rows + 1) / 2;
    for (size_t h = 0; h < heads; ++h)
        for (size_t row = 0; row < rows; ++row)
            for (size_t col = 0; col <= pos0 + row && col < seq; ++col) {
                int64_t acc = 0;
                for (size_t l = 0; l < head_dim; ++l)
                    acc += (int64_t)q[row * d + h * head_dim + l] * (int64_t)k[col * d + h * head_dim + l];
                const size_t p = h * per_head + packed_prefix(row, pos0) + col;
                accs[p] = acc;
                outs[p] = score_clamp17(acc, shift, err);
            }
}

/* backend.cu:1619-1634 */
static int16_t recip_value(int64_t input, const int16_t* lut, uint32_t den_shift, uint32_t recip_log2,
                           int use_row_shift, uint32_t* err) {
    const int64_t limit = use_row_shift ? ((int64_t)1 << 18) : ((int64_t)1 << 16);
    if (input < 0 || input >= limit) {
        *err = 1;
        return lut[0];
    }
    if (input < ((int64_t)1 << 16)) return lut[(size_t)input];
    const uint64_t den_back = ((uint64_t)input << den_shift) + ((uint64_t)1 << (den_shift - 1));
    uint64_t v = (((uint64_t)1 << recip_log2) + den_back / 2) / den_back;
    if (v > (uint64_t)INT16_MAX) v = INT16_MAX;
    return (int16_t)v;
}

/* backend.cu:1636-1687 */
void or_fixed_softmax(const int16_t* scores, const int16_t* exp_lut, const int16_t* recip_lut, int16_t* row_shifts,
                      int16_t* exp_out, int64_t* denoms, int16_t* recips, int16_t* weights, uint32_t* err,
                      size_t rows, size_t pos0, size_t heads, uint32_t recip_den_shift, uint32_t recip_log2,
                      uint32_t norm_shift, int use_row_shift) {
    const size_t per_head = rows * pos0 + rows * (rows + 1) / 2;
    for (size_t h = 0; h < heads; ++h)
        for (size_t row = 0; row < rows; ++row) {
            const size_t width = pos0 + row + 1;
            const size_t start = h * per_head + packed_prefix(row, pos0);
            int16_t sv = 0;
            if (use_row_shift) {
                sv = scores[start];
                for (size_t j = 1; j < width; ++j)
                    if (scores[start + j] > sv) sv = scores[start + j];
            }
            row_shifts[h * rows + row] = sv;
            int64_t denom = 0;
            for (size_t j = 0; j < width; ++j) {
                const int32_t s = scores[start + j];
                int16_t v = 0;
                if (use_row_shift) {
                    const int32_t gap = (int32_t)sv - s;
                    if (gap < 0 || gap > UINT16_MAX) {
                        *err = 1;
                    } else if (gap <= 32768) {
                        v = exp_lut[(uint16_t)(int16_t)(-gap)];
                    } else if (exp_lut[(uint16_t)INT16_MIN] != 0) {
                        *err = 1;
                    }
                } else {
                    v = exp_lut[(uint16_t)scores[start + j]];
                }
                exp_out[start + j] = v;
                denom += v;
            }
            const int64_t ri = denom >> recip_den_shift;
            const int16_t rc = recip_value(ri, recip_lut, recip_den_shift, recip_log2, use_row_shift, err);
            denoms[h * rows + row] = denom;
            recips[h * rows + row] = rc;
            for (size_t j = 0; j < width; ++j)
                weights[start + j] = requant_no_clamp((int64_t)exp_out[start + j] * rc, norm_shift, err);
        }
}

/* backend.cu:1689-1709 */
void or_fixed_av(const int16_t* weights, const int16_t* values, int64_t* accs, int16_t* outs, uint32_t* err,
                 size_t rows, size_t seq, size_t pos0, size_t d, size_t heads, uint32_t shift) {
    const size_t head_dim = d / heads;
    const size_t per_head = rows * pos0 + rows * (rows + 1) / 2;
    for (size_t row = 0; row < rows; ++row)
        for (size_t col = 0; col < d; ++col) {
            const size_t h = col / head_dim;
            const size_t width = pos0 + row + 1;
            const size_t start = h * per_head + packed_prefix(row, pos0);
            int64_t acc = 0;
            for (size_t j = 0; j < width; ++j) acc += (int64_t)weights[start + j] * (int64_t)values[j * d + col];
            accs[row * d + col] = acc;
            outs[row * d + col] = requant_no_clamp(acc, shift, err);
        }
}

/* backend.cu:1711-1724 */
void or_fixed_lookup(const int16_t* input, const int16_t* lut, int16_t* out, size_t n) {
    for (size_t z = 0; z < n; ++z) out[z] = lut[(uint16_t)input[z]];
}

void or_fixed_requant_i16(const int16_t* input, int16_t* out, uint32_t* err, size_t n, uint32_t shift) {
    for (size_t z = 0; z < n; ++z) out[z] = shift == 0 ? input[z] : requant_no_clamp(input[z], shift, err);
}

/* backend.cu:1726-1740: logits x wte^T, i64, no requant */
void or_fixed_logits(const int16_t* input, const int16_t* w, int64_t* out, size_t rows, size_t d, size_t vocab) {
#pragma omp parallel for schedule(static)
    for (size_t row = 0; row < rows; ++row)
        for (size_t word = 0; word < vocab; ++word) {
            int64_t acc = 0;
            for (size_t j = 0; j < d; ++j) acc += (int64_t)input[row * d + j] * (int64_t)w[word * d + j];
            out[row * vocab + word] = acc;
        }
}

/* ---- attention proof wires (backend.cu:2202-2470, 5278-5375) ---- */

/* backend.cu fp_from_i64_device: the canonical residue of a signed value */
static uint64_t fp_of_i64(int64_t v) {
    const uint64_t p = 0xFFFFFFFF00000001ull;
    if (v >= 0) return (uint64_t)v % p;
    const uint64_t mag = (uint64_t)(-(v + 1)) + 1, r = mag % p;
    return r == 0 ? 0 : p - r;
}

/* rect: 9 columns of head_pad x query_pad x seq_pad entries; above: the
 * strictly-above-causal full scores; rows: 13 columns of head_pad x
 * query_pad; qkv: 2 columns of query_pad x 4 d_pad. */
void or_attention_wires(const or_wires_geom* g, const int16_t* q, const int16_t* k_cache, const int16_t* own_k,
                        const int16_t* v, const int64_t* scores_acc, const int16_t* scores_q,
                        const int16_t* row_shifts, const int16_t* exp_outputs, const int64_t* denoms,
                        const int16_t* recips, const int16_t* weights, const int16_t* recip_lut,
                        const int64_t* qkv_acc, uint64_t* rect, uint64_t* rows_out, uint64_t* above,
                        uint64_t* qkv_cols, uint32_t* err) {
    const size_t qr = g->query_rows, d = g->heads * g->head_dim;
    const size_t per_head = qr * g->pos0 + qr * (qr + 1) / 2;
    const int rs = g->use_row_shift;
    /* rectangle columns */
    const size_t sp2 = g->query_pad * g->seq_pad, rect_n = g->head_pad * sp2;
    for (size_t z = 0; z < rect_n; ++z) {
        const size_t head = z / sp2, rem = z % sp2, row = rem / g->seq_pad, col = rem % g->seq_pad;
        const int64_t half_s = (int64_t)1 << (g->shift_scores - 1), half_n = (int64_t)1 << (g->shift_softmax_norm - 1);
        int64_t norm_rem = half_n, weight = 0, score_rem = half_s;
        int64_t score_value = rs ? -(int64_t)g->exp_pad_input : (int64_t)g->exp_pad_input;
        int64_t score_index = score_value + ((int64_t)1 << 16);
        int64_t exp_input = g->exp_pad_input, exp_value = 0, is_max = 0, full = 0;
        if (head < g->heads && row < qr && col < g->seq) {
            for (size_t l = 0; l < g->head_dim; ++l)
                full += (int64_t)q[row * d + head * g->head_dim + l] * (int64_t)k_cache[col * d + head * g->head_dim + l];
            const size_t width = g->pos0 + row + 1;
            if (col < width) {
                const size_t start = head * per_head + packed_prefix(row, g->pos0), pk = start + col;
                const int64_t score = scores_q[pk];
                const int64_t raw = requant_rounded(scores_acc[pk], g->shift_scores);
                const int64_t clamped = raw < INT16_MIN ? INT16_MIN : (raw > INT16_MAX ? INT16_MAX : raw);
                if (raw < -((int64_t)1 << 16) || raw >= ((int64_t)1 << 16) || score != clamped) *err = 1;
                const int64_t shift_v = rs ? row_shifts[head * qr + row] : 0;
                score_value = score;
                score_index = raw + ((int64_t)1 << 16);
                exp_input = rs ? shift_v - score : score;
                if ((rs && (exp_input < 0 || exp_input > UINT16_MAX)) ||
                    (!rs && (exp_input < INT16_MIN || exp_input > INT16_MAX)))
                    *err = 1;
                score_rem = scores_acc[pk] + half_s - raw * ((int64_t)1 << g->shift_scores);
                if (score_rem < 0 || score_rem >= ((int64_t)1 << g->shift_scores)) *err = 1;
                if (scores_acc[pk] != full) *err = 1;
                exp_value = exp_outputs[pk];
                weight = weights[pk];
                const int64_t rc = recips[head * qr + row];
                norm_rem = exp_value * rc + half_n - weight * ((int64_t)1 << g->shift_softmax_norm);
                if (norm_rem < 0 || norm_rem >= ((int64_t)1 << g->shift_softmax_norm)) *err = 1;
                if (rs && exp_input == 0) {
                    int first = 1;
                    for (size_t prior = 0; prior < col; ++prior)
                        if ((int64_t)scores_q[start + prior] - shift_v == 0) {
                            first = 0;
                            break;
                        }
                    is_max = first;
                }
            } else {
                const size_t local = col - width;
                const size_t row_prefix = row * (qr - 1) - row * (row - 1) / 2;
                above[head * (qr * (qr - 1) / 2) + row_prefix + local] = fp_of_i64(full);
            }
        }
        rect[z] = (uint64_t)norm_rem;
        rect[rect_n + z] = fp_of_i64(weight);
        rect[2 * rect_n + z] = (uint64_t)score_rem;
        rect[3 * rect_n + z] = rs ? (uint64_t)score_index : fp_of_i64(score_value);
        rect[4 * rect_n + z] = fp_of_i64(score_value);
        rect[5 * rect_n + z] = rs ? (uint64_t)exp_input : fp_of_i64(exp_input);
        rect[6 * rect_n + z] = fp_of_i64(exp_value);
        rect[7 * rect_n + z] = (uint64_t)is_max;
        rect[8 * rect_n + z] = fp_of_i64(full);
    }
    /* row columns */
    const size_t row_n = g->head_pad * g->query_pad;
    for (size_t z = 0; z < row_n; ++z) {
        const size_t head = z / g->query_pad, row = z % g->query_pad;
        int64_t denom = 0, rin = 0, rc = g->recip_pad_output, shift_v = 0;
        int real = 0;
        if (head < g->heads && row < qr) {
            real = 1;
            denom = denoms[head * qr + row];
            rin = denom >> g->recip_den_shift;
            rc = recips[head * qr + row];
            shift_v = rs ? row_shifts[head * qr + row] : 0;
            if (recip_value(rin, recip_lut, g->recip_den_shift, g->recip_log2, rs, err) != rc) *err = 1;
            if (rs) {
                const size_t start = head * per_head + packed_prefix(row, g->pos0), width = g->pos0 + row + 1;
                int found = 0;
                for (size_t c = 0; c < width; ++c)
                    if (scores_q[start + c] == shift_v) {
                        found = 1;
                        break;
                    }
                if (!found || width > g->seq) *err = 1;
            }
        }
        rows_out[z] = fp_of_i64(denom);
        rows_out[row_n + z] = (uint64_t)rin;
        rows_out[2 * row_n + z] = fp_of_i64(rc);
        rows_out[3 * row_n + z] = fp_of_i64(shift_v);
        const uint32_t ds = g->recip_den_shift;
        const int64_t r_in = real ? rin : 256;
        const int64_t r_den = real ? denom : ((int64_t)256 << ds);
        const int64_t r_q = real ? rc : recip_value(256, recip_lut, ds, g->recip_log2, 1, err);
        const int64_t denom_low = r_den - (r_in << ds);
        const int64_t divisor = (r_in << ds) + ((int64_t)1 << (ds - 1));
        const int64_t numer = ((int64_t)1 << g->recip_log2) + divisor / 2;
        const int64_t remainder = numer - r_q * divisor;
        const int64_t slack = divisor - 1 - remainder;
        if (denom_low < 0 || denom_low >= ((int64_t)1 << ds) || r_in < 0 || r_in >= ((int64_t)1 << 18) || r_q < 0 ||
            r_q >= ((int64_t)1 << 15) || remainder < 0 || remainder >= divisor || remainder >= ((int64_t)1 << 24) ||
            slack < 0 || slack >= ((int64_t)1 << 24))
            *err = 1;
        rows_out[4 * row_n + z] = (uint64_t)denom_low;
        rows_out[5 * row_n + z] = (uint64_t)(r_in & 0xffff);
        rows_out[6 * row_n + z] = (uint64_t)(r_in >> 16);
        rows_out[7 * row_n + z] = (uint64_t)r_q;
        rows_out[8 * row_n + z] = (uint64_t)(remainder & 0xffff);
        rows_out[9 * row_n + z] = (uint64_t)(remainder >> 16);
        rows_out[10 * row_n + z] = (uint64_t)(slack & 0xffff);
        rows_out[11 * row_n + z] = (uint64_t)(slack >> 16);
        rows_out[12 * row_n + z] = (uint64_t)divisor;
    }
    /* QKV requant columns */
    const size_t width = 4 * g->d_pad, qkv_n = g->query_pad * width;
    for (size_t z = 0; z < qkv_n; ++z) {
        const size_t row = z / width, col = z % width, third = col / g->d_pad, rest = col % g->d_pad;
        const int64_t half = (int64_t)1 << (g->shift_qkv - 1);
        int64_t rem = half, out = 0;
        if (row < qr && third < 3 && rest < d) {
            out = third == 0 ? q[row * d + rest] : (third == 1 ? own_k[row * d + rest] : v[row * d + rest]);
            rem = qkv_acc[row * 3 * d + third * d + rest] + half - out * ((int64_t)1 << g->shift_qkv);
            if (rem < 0 || rem >= ((int64_t)1 << g->shift_qkv)) *err = 1;
        }
        qkv_cols[z] = (uint64_t)rem;
        qkv_cols[qkv_n + z] = fp_of_i64(out);
    }
}
