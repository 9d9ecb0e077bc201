/*
 * CPU ORACLE — TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the arithmetic of the comfyui-turing-utils quantized
 * DiT path (ConvRot activation quantizer, INT8 GEMM accumulate + dequant
 * epilogue, W4 / codebook-W4 weight decode, Sage Q/K INT8 quantizer).  Only the
 * test suite, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
 * arm load this file; the product path never does.
 *
 * Every function names the reference file:line it restates (paths are relative
 * to the reference project root).  Compile with -ffp-contract=off and without
 * -ffast-math: the reference's `_C` extension is built without fast-math
 * (kernel/setup.py:398-412), so its divides and adds are IEEE round-to-nearest
 * and the order of every floating-point operation below matters.
 */
#include <math.h>
#include <stdlib.h>
#include <stdint.h>
#include <string.h>

/* ---------------------------------------------------------------- bf16 --- */

/* kernel/csrc/turing/convrot_quant.cu:293-305 (float_to_bf16_rn_bits) */
static inline uint16_t f32_to_bf16_rn(float v) {
    uint32_t bits;
    memcpy(&bits, &v, 4);
    if ((bits & 0x7fffffffu) > 0x7f800000u) return 0x7fffu;
    uint16_t upper = (uint16_t)(bits >> 16);
    uint32_t rem = bits << 16;
    if (rem > 0x80000000u || (rem == 0x80000000u && (upper & 1u))) ++upper;
    return upper;
}

static inline float bf16_to_f32(uint16_t h) {
    uint32_t bits = ((uint32_t)h) << 16;
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* IEEE binary16 <-> binary32 (round to nearest even), used for FP16 inputs of
 * the staged quantizer (convrot_quant.cu:33-54) and for E4M3 decode. */
static inline float f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    int exp = (h >> 10) & 0x1f;
    uint32_t mant = h & 0x3ffu;
    uint32_t bits;
    if (exp == 0) {
        if (mant == 0) {
            bits = sign;
        } else {
            int e = -1;
            do { mant <<= 1; ++e; } while (!(mant & 0x400u));
            mant &= 0x3ffu;
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (mant << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7f800000u | (mant << 13);
    } else {
        bits = sign | ((uint32_t)(exp - 15 + 127) << 23) | (mant << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static inline uint16_t f32_to_f16_rn(float v) {
    uint32_t bits;
    memcpy(&bits, &v, 4);
    uint32_t sign = (bits >> 16) & 0x8000u;
    uint32_t absb = bits & 0x7fffffffu;
    if (absb > 0x7f800000u) return (uint16_t)(sign | 0x7e00u);
    if (absb >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* rounds to inf */
    if (absb < 0x38800000u) {                                   /* subnormal f16 */
        if (absb < 0x33000000u) return (uint16_t)sign;           /* < 2^-25 -> 0 */
        int e = (int)(absb >> 23);
        uint32_t m = (absb & 0x7fffffu) | 0x800000u;
        int shift = 126 - e; /* q = m * 2^(e-126): value in units of 2^-24 */
        uint32_t q = m >> shift;
        uint32_t r = m & ((1u << shift) - 1u);
        uint32_t half = 1u << (shift - 1);
        if (r > half || (r == half && (q & 1u))) ++q;
        return (uint16_t)(sign | q);
    }
    uint32_t e = (absb >> 23) - 112;
    uint32_t m = absb & 0x7fffffu;
    uint32_t q = (e << 10) | (m >> 13);
    uint32_t r = m & 0x1fffu;
    if (r > 0x1000u || (r == 0x1000u && (q & 1u))) ++q;
    return (uint16_t)(sign | q);
}

/* E4M3 (OCP fp8, no infinities, 0x7f/0xff NaN) -> float.  Every finite E4M3
 * value is exact in half and float, so this equals the reference's
 * __nv_cvt_fp8_to_halfraw(value, __NV_E4M3) -> __half2float
 * (kernel/csrc/turing/w4a8.cu:77-80). */
float orc_e4m3_to_f32(uint8_t v) {
    int sign = v >> 7;
    int exp = (v >> 3) & 0xf;
    int mant = v & 7;
    float out;
    if (exp == 15 && mant == 7) {
        out = NAN;
    } else if (exp == 0) {
        out = ldexpf((float)mant, -9);
    } else {
        out = ldexpf((float)(8 + mant), exp - 10);
    }
    return sign ? -out : out;
}

/* ------------------------------------------------------------- ConvRot --- */

#define GROUP 256

/* One radix-4 stage of the 256-point block Hadamard, in the reference's exact
 * per-output operation order: kernel/csrc/turing/convrot_quant.cu:104-116
 * (fht_stage) and :385-391 (the S=1 stage fused with the load). */
static void fht_stage(const float *src, float *dst, int S) {
    for (int lane = 0; lane < 64; ++lane) {
        int base = (lane % S) + (lane / S) * (4 * S);
        float x0 = src[base], x1 = src[base + S], x2 = src[base + 2 * S], x3 = src[base + 3 * S];
        dst[base] = 0.5f * (x0 + x1 + x2 - x3);
        dst[base + S] = 0.5f * (x0 + x1 - x2 + x3);
        dst[base + 2 * S] = 0.5f * (x0 - x1 + x2 + x3);
        dst[base + 3 * S] = 0.5f * (-x0 + x1 + x2 + x3);
    }
}

/* Rotate one 256-group of fp32 inputs: stages S = 1, 4, 16, 64 in that order
 * (convrot_quant.cu:384-403).  Returns the fp32 rotated values in y. */
static void fht256(const float *x, float *y) {
    float a[GROUP], b[GROUP];
    fht_stage(x, a, 1);
    fht_stage(a, b, 4);
    fht_stage(b, a, 16);
    fht_stage(a, y, 64);
}

/* SwiGLU load: convrot_quant.cu:137-143.  expf is the C library's, so this
 * can differ from CUDA's expf in the last place; tests of the fused variants
 * therefore allow rare +-1 code differences (documented in the tests). */
static inline float swiglu_f(float gate, float up) {
    return (gate / (1.0f + expf(-gate))) * up;
}

/* tanh-GELU load rounded to the input dtype: convrot_quant.cu:145-156.  The
 * inner x + beta*x^3 is written as the FMA that nvcc's default contraction
 * forms from the reference expression. */
static inline float gelu_f(float x, int fp16_input) {
    const float kAlpha = 0.7978845608028654f;
    const float kBeta = 0.044715f;
    float inner = fmaf(kBeta * x * x, x, x);
    float act = 0.5f * x * (1.0f + tanhf(kAlpha * inner));
    return fp16_input ? f16_to_f32(f32_to_f16_rn(act)) : bf16_to_f32(f32_to_bf16_rn(act));
}

/* ConvRot activation quantizer.
 *   input : [rows, act==1 ? 2k : k] of bf16 (in_fp16=0) or fp16 (in_fp16=1)
 *   act   : 0 none, 1 SwiGLU (gate = first half, up = second half), 2 tanh-GELU
 *   int4  : 0 -> out int8 [rows, k];  1 -> packed int4 [rows, k/2] (low = even col)
 *   staged: 0 -> BF16 row-buffer kernel (convrot_quant.cu:350-444)
 *           1 -> staged two-kernel path (convrot_quant.cu:158-291)
 *   scales: [rows] fp32
 * The two forms differ only in how the per-row scale is formed
 * (staged: min(amax,max)*(1/127); row-buffer: min(amax,max)/127) and in the
 * staged path's FP16 scratch for FP16 inputs.
 */
void orc_convrot_quantize(const uint16_t *input, int64_t rows, int64_t k, int act, int int4,
                          int staged, int in_fp16, int8_t *out, float *scales) {
    const int64_t in_width = act == 1 ? 2 * k : k;
    const int groups = (int)(k / GROUP);
    float xin[GROUP], y[GROUP];
    uint16_t *buf = (uint16_t *)malloc((size_t)k * sizeof(uint16_t));
    for (int64_t row = 0; row < rows; ++row) {
        const uint16_t *src = input + row * in_width;
        float amax = 0.0f;
        for (int g = 0; g < groups; ++g) {
            for (int i = 0; i < GROUP; ++i) {
                int64_t col = (int64_t)g * GROUP + i;
                float v;
                if (act == 1) {
                    float gate = in_fp16 ? f16_to_f32(src[col]) : bf16_to_f32(src[col]);
                    float up = in_fp16 ? f16_to_f32(src[k + col]) : bf16_to_f32(src[k + col]);
                    v = swiglu_f(gate, up);
                } else if (act == 2) {
                    float x = in_fp16 ? f16_to_f32(src[col]) : bf16_to_f32(src[col]);
                    v = gelu_f(x, in_fp16);
                } else {
                    v = in_fp16 ? f16_to_f32(src[col]) : bf16_to_f32(src[col]);
                }
                xin[i] = v;
            }
            fht256(xin, y);
            for (int i = 0; i < GROUP; ++i) {
                /* fht_store_bf16_absmax: store the rounded value, take the
                 * absmax of the fp32 value (convrot_quant.cu:311-330). */
                buf[(int64_t)g * GROUP + i] = in_fp16 ? f32_to_f16_rn(y[i]) : f32_to_bf16_rn(y[i]);
                amax = fmaxf(amax, fabsf(y[i]));
            }
        }
        const float fmax_in = in_fp16 ? 65504.0f : 3.38953139e38f;
        const float qmax = int4 ? 7.0f : 127.0f;
        const float floor_v = int4 ? 1.0e-10f : 1.0e-30f;
        float clipped = fminf(amax, fmax_in);
        float scale = staged ? fmaxf(clipped * (1.0f / qmax), floor_v)
                             : fmaxf(clipped / qmax, floor_v);
        scales[row] = scale;
        if (int4) {
            /* convrot_quant.cu:418-433 / :280-290 */
            const float inv = 1.0f / scale;
            int8_t *dst = out + row * (k / 2);
            for (int64_t pc = 0; pc < k / 2; ++pc) {
                float lo_v = in_fp16 ? f16_to_f32(buf[2 * pc]) : bf16_to_f32(buf[2 * pc]);
                float hi_v = in_fp16 ? f16_to_f32(buf[2 * pc + 1]) : bf16_to_f32(buf[2 * pc + 1]);
                float lo = nearbyintf(lo_v * inv);
                float hi = nearbyintf(hi_v * inv);
                lo = fminf(7.0f, fmaxf(-7.0f, lo));
                hi = fminf(7.0f, fmaxf(-7.0f, hi));
                uint8_t lb = (uint8_t)((int8_t)lo) & 0x0f;
                uint8_t hb = (uint8_t)((int8_t)hi) & 0x0f;
                dst[pc] = (int8_t)(lb | (hb << 4));
            }
        } else {
            /* convrot_quant.cu:417,434-442 / :69-73,242-247 */
            float rs = in_fp16 ? f16_to_f32(f32_to_f16_rn(scale)) : bf16_to_f32(f32_to_bf16_rn(scale));
            int8_t *dst = out + row * k;
            for (int64_t c = 0; c < k; ++c) {
                float v = in_fp16 ? f16_to_f32(buf[c]) : bf16_to_f32(buf[c]);
                float d = v / rs;
                d = in_fp16 ? f16_to_f32(f32_to_f16_rn(d)) : bf16_to_f32(f32_to_bf16_rn(d));
                float q = nearbyintf(d);
                q = fminf(127.0f, fmaxf(-128.0f, q));
                dst[c] = (int8_t)q;
            }
        }
    }
    free(buf);
}

/* Rotated bf16 values only (the staged kernel's `rotated` scratch,
 * convrot_quant.cu:158-211), for diagnostics. */
void orc_convrot_rotate_bf16(const uint16_t *input, int64_t rows, int64_t k, uint16_t *out,
                             float *group_absmax) {
    const int groups = (int)(k / GROUP);
    float xin[GROUP], y[GROUP];
    for (int64_t row = 0; row < rows; ++row) {
        for (int g = 0; g < groups; ++g) {
            float am = 0.0f;
            for (int i = 0; i < GROUP; ++i) xin[i] = bf16_to_f32(input[row * k + (int64_t)g * GROUP + i]);
            fht256(xin, y);
            for (int i = 0; i < GROUP; ++i) {
                out[row * k + (int64_t)g * GROUP + i] = f32_to_bf16_rn(y[i]);
                am = fmaxf(am, fabsf(y[i]));
            }
            group_absmax[row * groups + g] = am;
        }
    }
}

/* ------------------------------------------------------- INT8 GEMM ------- */

/* acc[m, n] = sum_k A[m, k] * W[n, k] in exact integer arithmetic
 * (kernel/csrc/turing/w4a8.cu:376-418: S8 x S8 -> S32, OpMultiplyAddSaturate;
 * with |acc| <= 127*128*K no saturation occurs for K < 132,000). Rows given by
 * row_index (so tests can sample rows of a large problem); n_rows rows out. */
void orc_int8_gemm_rows(const int8_t *A, const int8_t *W, int64_t N, int64_t K,
                        const int64_t *row_index, int64_t n_rows, int32_t *acc) {
    for (int64_t r = 0; r < n_rows; ++r) {
        const int8_t *a = A + row_index[r] * K;
        for (int64_t n = 0; n < N; ++n) {
            const int8_t *w = W + n * K;
            int32_t s = 0;
            for (int64_t k = 0; k < K; ++k) s += (int32_t)a[k] * (int32_t)w[k];
            acc[r * N + n] = s;
        }
    }
}

/* Dequantize epilogue: v = ((float)acc * a_s[m]) * w_s[n] (+ bias[n]) -> bf16 RNE.
 * Operation order of kernel/csrc/turing/bf16_epilogue.cu:105-119 and of the
 * GEMM EVT tree w4a8.cu:474-525 (multiply by the row scale, then the column
 * scale, then add the bias).  The add is a separate rounding here (no FMA);
 * the CUDA epilogue in this repository uses the same two-step form.
 * w_scalar: weight_scale has one element (bf16_epilogue.cu:81-89). */
void orc_dequant_bf16(const int32_t *acc, int64_t rows, int64_t cols, int64_t acc_stride,
                      const float *a_s, const float *w_s, int w_scalar, const float *bias,
                      uint16_t *out) {
    for (int64_t m = 0; m < rows; ++m) {
        for (int64_t n = 0; n < cols; ++n) {
            float v = (float)acc[m * acc_stride + n] * a_s[m];
            v = v * (w_scalar ? w_s[0] : w_s[n]);
            if (bias) v = v + bias[n];
            out[m * cols + n] = f32_to_bf16_rn(v);
        }
    }
}

/* ------------------------------------------------------ weight decode ---- */

/* Legacy signed-nibble W4: low nibble = even k, sign extended
 * (w4a8.cu:34-72, validate_compatible.py:28-40). packed [N, K/2] -> int8 [N, K]. */
void orc_unpack_int4(const int8_t *packed, int64_t n, int64_t k, int8_t *out) {
    for (int64_t r = 0; r < n; ++r) {
        for (int64_t j = 0; j < k / 2; ++j) {
            uint8_t b = (uint8_t)packed[r * (k / 2) + j];
            int lo = b & 0xf, hi = b >> 4;
            if (lo >= 8) lo -= 16;
            if (hi >= 8) hi -= 16;
            out[r * k + 2 * j] = (int8_t)lo;
            out[r * k + 2 * j + 1] = (int8_t)hi;
        }
    }
}

/* Grouped-codebook W4 decode (w4a8.cu:907-973, iterator :209-223):
 * w8[n,k] = clamp(rint_even(codebook[idx] * float(e4m3(group_scale[n, k/g]))), -127, 127).
 * idx: low nibble = even column. */
void orc_codebook_decode(const int8_t *packed, const uint8_t *group_scale, const float *codebook,
                         int64_t n, int64_t k, int64_t group_size, int8_t *out) {
    const int64_t gpr = k / group_size;
    for (int64_t r = 0; r < n; ++r) {
        for (int64_t c = 0; c < k; ++c) {
            uint8_t b = (uint8_t)packed[r * (k / 2) + c / 2];
            int code = (c & 1) ? (b >> 4) : (b & 0xf);
            float s = orc_e4m3_to_f32(group_scale[r * gpr + c / group_size]);
            float v = codebook[code] * s;
            float q = nearbyintf(v);
            if (q > 127.0f) q = 127.0f;
            if (q < -127.0f) q = -127.0f;
            out[r * k + c] = (int8_t)q;
        }
    }
}

/* ----------------------------------------------------------- Sage quant -- */

/* cvt.rni.sat.s8.f32: round to nearest even, saturate, NaN -> 0
 * (kernel/csrc/turing/sage/numeric_conversion.cuh:144-149). */
static inline int8_t cvt_rni_sat_s8(float x) {
    if (isnan(x)) return 0;
    float r = nearbyintf(x);
    if (r > 127.0f) r = 127.0f;
    if (r < -128.0f) r = -128.0f;
    return (int8_t)r;
}

/* Per-tile INT8 quantizer QuantInt8Kernel (kernel/csrc/turing/sage/fused.cu:66-200).
 * x is [tiles_outer, L, D] with arbitrary strides given in elements:
 *   element (o, t, d) at x[o*s_outer + t*s_tok + d]; out uses the same
 *   strides (the reference requires contiguous outputs with the input shape).
 * tile tokens T (16 = Q per-warp, 64 = K per-block).  scale [outer, tiles].
 * mean (optional, bf16/f16 bits, [outer, D] with stride s_mean_outer): the
 * sub_mean branch (fused.cu:97-128), subtracted in fp32.
 * Division semantics: the reference extension is built with --use_fast_math;
 * this oracle fixes IEEE 127/amax and amax/127 (see the module docstring). */
void orc_sage_quant(const uint16_t *x, int in_fp16, int64_t outer, int64_t L, int64_t D,
                    int64_t s_outer, int64_t s_tok, int64_t T, int64_t tiles,
                    const uint16_t *mean, int64_t s_mean_outer, int8_t *out, float *scale) {
    /* tiles >= ceil(L/T): the per-warp Q layout pads to whole 64-token blocks
     * and stores a scale for every warp tile (empty ones: 1e-7 / 127). */
    for (int64_t o = 0; o < outer; ++o) {
        for (int64_t t = 0; t < tiles; ++t) {
            float amax = 0.0000001f;
            for (int64_t i = 0; i < T; ++i) {
                int64_t tok = t * T + i;
                if (tok >= L) break;
                for (int64_t d = 0; d < D; ++d) {
                    uint16_t h = x[o * s_outer + tok * s_tok + d];
                    float v = in_fp16 ? f16_to_f32(h) : bf16_to_f32(h);
                    if (mean) {
                        uint16_t mh = mean[o * s_mean_outer + d];
                        v -= in_fp16 ? f16_to_f32(mh) : bf16_to_f32(mh);
                    }
                    amax = fmaxf(amax, fabsf(v));
                }
            }
            scale[o * tiles + t] = amax / 127.0f;
            float tmp = 127.0f / amax;
            for (int64_t i = 0; i < T; ++i) {
                int64_t tok = t * T + i;
                if (tok >= L) break;
                for (int64_t d = 0; d < D; ++d) {
                    uint16_t h = x[o * s_outer + tok * s_tok + d];
                    float v = in_fp16 ? f16_to_f32(h) : bf16_to_f32(h);
                    if (mean) {
                        uint16_t mh = mean[o * s_mean_outer + d];
                        v -= in_fp16 ? f16_to_f32(mh) : bf16_to_f32(mh);
                    }
                    out[o * s_outer + tok * s_tok + d] = cvt_rni_sat_s8(v * tmp);
                }
            }
        }
    }
}

/* K smoothing mean over tokens, per (outer, channel): accumulated in double,
 * divided by L, rounded to float and then to the input dtype.  The sum is in
 * double so that the value does not depend on the summation order the CUDA
 * kernel uses (it also accumulates in double). */
void orc_token_mean(const uint16_t *x, int in_fp16, int64_t outer, int64_t L, int64_t D,
                    int64_t s_outer, int64_t s_tok, uint16_t *mean) {
    for (int64_t o = 0; o < outer; ++o) {
        for (int64_t d = 0; d < D; ++d) {
            double s = 0.0;
            for (int64_t t = 0; t < L; ++t) {
                uint16_t h = x[o * s_outer + t * s_tok + d];
                s += (double)(in_fp16 ? f16_to_f32(h) : bf16_to_f32(h));
            }
            float m = (float)(s / (double)L);
            mean[o * D + d] = in_fp16 ? f32_to_f16_rn(m) : f32_to_bf16_rn(m);
        }
    }
}

/* ------------------------------------------ fused RMSNorm + RoPE + INT8 -- */

/* Correctly rounded 1/sqrt(y) for y > 0 (the value __frsqrt_rn returns):
 * formed in double, whose 29 extra bits leave a wrong final rounding only
 * when 1/sqrt(y) lies within 2^-53 (relative) of a float rounding boundary. */
static inline float rsqrt_rn(float y) { return (float)(1.0 / sqrt((double)y)); }

static inline float round_elem(float v, int fp16) {
    return fp16 ? f16_to_f32(f32_to_f16_rn(v)) : bf16_to_f32(f32_to_bf16_rn(v));
}

static inline float elem(const uint16_t *p, int64_t i, int fp16) {
    return fp16 ? f16_to_f32(p[i]) : bf16_to_f32(p[i]);
}

/* Row-scope RRMS of token (b, tok) over all H heads, summed in the CUDA
 * block's order (kernel/csrc/turing/sage/qk_preprocess.cu:203-251 with
 * reduction_utils.cuh:70-87): 256 per-thread FMA chains over i = h*D + c
 * strided by 256, an XOR butterfly inside each 32-lane warp, then an XOR
 * butterfly over the 8 warp partials padded with zeros to 32 lanes. */
static float row_rrms(const uint16_t *x, int64_t H, int64_t L, int64_t D, int64_t b,
                      int64_t tok, int fp16, float eps) {
    float lanes[256], w[32];
    const int64_t n = H * D;
    for (int t = 0; t < 256; ++t) {
        float s = 0.0f;
        for (int64_t i = t; i < n; i += 256) {
            const int64_t h = i / D, c = i - h * D;
            const float v = elem(x, ((b * H + h) * L + tok) * D + c, fp16);
            s = fmaf(v, v, s);
        }
        lanes[t] = s;
    }
    for (int wp = 0; wp < 8; ++wp) {
        float *l = lanes + wp * 32, tmp[32];
        for (int o = 16; o > 0; o >>= 1) {
            for (int i = 0; i < 32; ++i) tmp[i] = l[i] + l[i ^ o];
            memcpy(l, tmp, sizeof(tmp));
        }
        w[wp] = l[0];
    }
    for (int i = 8; i < 32; ++i) w[i] = 0.0f;
    for (int o = 16; o > 0; o >>= 1) {
        float tmp[32];
        for (int i = 0; i < 32; ++i) tmp[i] = w[i] + w[i ^ o];
        memcpy(w, tmp, sizeof(tmp));
    }
    return rsqrt_rn(w[0] / (float)n + eps);
}

/* Head-scope RRMS of one token row (qk_preprocess.cu:505-515): an 8-channel
 * FMA chain per pack, then an XOR butterfly over the D/8 packs. */
static float head_rrms(const uint16_t *row, int64_t D, int fp16, float eps) {
    float p[16], tmp[16];
    const int P = (int)(D / 8);
    for (int k = 0; k < P; ++k) {
        float s = 0.0f;
        for (int c = 0; c < 8; ++c) {
            const float v = elem(row, k * 8 + c, fp16);
            s = fmaf(v, v, s);
        }
        p[k] = s;
    }
    for (int o = P / 2; o > 0; o >>= 1) {
        for (int i = 0; i < P; ++i) tmp[i] = p[i] + p[i ^ o];
        memcpy(p, tmp, sizeof(float) * (size_t)P);
    }
    return rsqrt_rn(p[0] / (float)D + eps);
}

/* Fused RMSNorm + RoPE + per-tile INT8 quantization of one of Q/K
 * (qk_preprocess.cu:151-201 per element, :417-563 per tile).
 * x: [B, H, L, D] contiguous bits; norm: [D] (head scope) or [H*D] (row);
 * freqs: [fb, fs, rot_dim/2, 2, 2] contiguous bits or NULL (rot_dim 0).
 * T tokens per tile, tiles scale entries per (b, h) (empty tiles get the
 * 1e-7 floor).  Per element: n = T(x * rrms * w); RoPE pairs (2p, 2p+1) or,
 * split-half, (p, p + rot_dim/2): v = T(fma(f[row][1], n1, f[row][0] * n0));
 * per tile amax = max(1e-7, max|v|), scale = amax / 127,
 * q = clamp(rint(v * (127 / amax)), -127, 127), IEEE divides. */
/* The processed row of token tok of head h (qk_preprocess.cu:151-201):
 * n = T(x * rrms * w) per channel, then RoPE on the first rot_dim channels,
 * v = T(fma(f[row][1], n(second), f[row][0] * n(first))).  nrm: D scratch. */
static void process_row(const uint16_t *row, const uint16_t *w, const uint16_t *freqs, int64_t b,
                        int64_t tok, int64_t D, int64_t fb, int64_t fs, int rot_dim,
                        int split_half, int fp16, float rrms, float *nrm, float *v) {
    const int half = rot_dim / 2;
    for (int64_t c = 0; c < D; ++c)
        nrm[c] = round_elem(elem(row, c, fp16) * rrms * elem(w, c, fp16), fp16);
    for (int64_t c = 0; c < D; ++c) {
        v[c] = nrm[c];
        if (c < rot_dim) {
            const int64_t pair = split_half ? (c < half ? c : c - half) : c / 2;
            const int64_t first = split_half ? pair : 2 * pair;
            const int64_t second = split_half ? pair + half : first + 1;
            const int64_t comp = split_half ? (c >= half) : (c & 1);
            const int64_t fbase =
                (((fb == 1 ? 0 : b) * fs + (fs == 1 ? 0 : tok)) * half + pair) * 4 + comp * 2;
            const float f0 = elem(freqs, fbase, fp16);
            const float f1 = elem(freqs, fbase + 1, fp16);
            v[c] = round_elem(fmaf(f1, nrm[second], f0 * nrm[first]), fp16);
        }
    }
}

/* The normalized + rotated values of every token (the first half of the
 * fused prologue), written as T bits in the input's [B, H, L, D] layout. */
void orc_qk_processed(const uint16_t *x, const uint16_t *norm, const uint16_t *freqs, int64_t B,
                      int64_t H, int64_t L, int64_t D, int64_t fb, int64_t fs, int rot_dim,
                      int split_half, int row_scope, int fp16, float eps, uint16_t *out) {
    float *nrm = (float *)malloc(sizeof(float) * (size_t)D);
    float *v = (float *)malloc(sizeof(float) * (size_t)D);
    for (int64_t b = 0; b < B; ++b)
        for (int64_t h = 0; h < H; ++h)
            for (int64_t tok = 0; tok < L; ++tok) {
                const uint16_t *row = x + ((b * H + h) * L + tok) * D;
                const float rrms = row_scope ? row_rrms(x, H, L, D, b, tok, fp16, eps)
                                             : head_rrms(row, D, fp16, eps);
                process_row(row, norm + (row_scope ? h * D : 0), freqs, b, tok, D, fb, fs,
                            rot_dim, split_half, fp16, rrms, nrm, v);
                uint16_t *o = out + ((b * H + h) * L + tok) * D;
                for (int64_t c = 0; c < D; ++c) o[c] = fp16 ? f32_to_f16_rn(v[c]) : f32_to_bf16_rn(v[c]);
            }
    free(nrm);
    free(v);
}

void orc_qk_rms_rope(const uint16_t *x, const uint16_t *norm, const uint16_t *freqs, int64_t B,
                     int64_t H, int64_t L, int64_t D, int64_t T, int64_t tiles, int64_t fb,
                     int64_t fs, int rot_dim, int split_half, int row_scope, int fp16, float eps,
                     int8_t *out, float *scale) {
    float *vals = (float *)malloc(sizeof(float) * (size_t)(T * D));
    float *nrm = (float *)malloc(sizeof(float) * (size_t)D);
    for (int64_t b = 0; b < B; ++b) {
        for (int64_t h = 0; h < H; ++h) {
            const uint16_t *w = norm + (row_scope ? h * D : 0);
            for (int64_t t = 0; t < tiles; ++t) {
                float amax = 0.0000001f;
                for (int64_t i = 0; i < T; ++i) {
                    const int64_t tok = t * T + i;
                    if (tok >= L) break;
                    const uint16_t *row = x + ((b * H + h) * L + tok) * D;
                    const float rrms = row_scope ? row_rrms(x, H, L, D, b, tok, fp16, eps)
                                                 : head_rrms(row, D, fp16, eps);
                    process_row(row, w, freqs, b, tok, D, fb, fs, rot_dim, split_half, fp16, rrms,
                                nrm, vals + i * D);
                    for (int64_t c = 0; c < D; ++c) amax = fmaxf(amax, fabsf(vals[i * D + c]));
                }
                scale[(b * H + h) * tiles + t] = amax / 127.0f;
                const float inv = 127.0f / amax;
                for (int64_t i = 0; i < T; ++i) {
                    const int64_t tok = t * T + i;
                    if (tok >= L) break;
                    for (int64_t c = 0; c < D; ++c) {
                        const float r = nearbyintf(vals[i * D + c] * inv);
                        out[((b * H + h) * L + tok) * D + c] =
                            (int8_t)fminf(127.0f, fmaxf(-127.0f, r));
                    }
                }
            }
        }
    }
    free(vals);
    free(nrm);
}

/* ------------------------------------------------ W8A8-PV attention ---- */

/* Sign of channel c in the shared randomized Hadamard transform of Q and K
 * (kernel/csrc/turing/sage/fused.cu:201-213): bit c of the 128-bit sign word,
 * clear = negate.  The table is part of the format: Q/K codes depend on it. */
static const uint32_t kRotSigns[4] = {0x1035997bu, 0x8087f5eeu, 0xee2e4e1au, 0x71132418u};

static inline int rot_negative(int c) { return ((kRotSigns[c >> 5] >> (c & 31)) & 1u) == 0u; }

/* In-place randomized Walsh-Hadamard transform of one D-channel row (D = 64 or
 * 128) in the reference's operation order (fused.cu:215-258): signs, then the
 * butterflies of channel bits 0, 1, 2 (inside an 8-channel pack) and 3.. (across
 * packs), each stage lo' = lo + hi, hi' = lo - hi, then one multiply by
 * 1/sqrt(D) (0.125 or 0.08838834764831845f). */
static void rot_row(float *v, int D) {
    for (int c = 0; c < D; ++c)
        if (rot_negative(c)) v[c] = -v[c];
    for (int span = 1; span < D; span <<= 1) {
        for (int base = 0; base < D; base += 2 * span) {
            for (int o = 0; o < span; ++o) {
                const float lo = v[base + o], hi = v[base + o + span];
                v[base + o] = lo + hi;
                v[base + o + span] = lo - hi;
            }
        }
    }
    const float norm = D == 64 ? 0.125f : 0.08838834764831845f;
    for (int c = 0; c < D; ++c) v[c] *= norm;
}

/* Sum / max over the 32 lanes of a warp by the shfl_down tree (offsets 16, 8,
 * 4, 2, 1) as lane 0 sees it; lanes without a partner keep their own value. */
static float warp_tree(const float *lane_vals, int is_max) {
    float a[32];
    memcpy(a, lane_vals, sizeof(a));
    for (int off = 16; off > 0; off >>= 1) {
        float b[32];
        for (int i = 0; i < 32; ++i) {
            const float other = i + off < 32 ? a[i + off] : a[i];
            b[i] = is_max ? fmaxf(a[i], other) : a[i] + other;
        }
        memcpy(a, b, sizeof(a));
    }
    return a[0];
}

/* Anchor choice over nine sampled key rows samp[9][128] of one (batch, kv head)
 * (DetectKAnchorKernel, fused.cu:406-556; detect_anchor_kernel,
 * qk_preprocess.cu:252-415, the same statistics): the sample nearest the
 * samples' mean (squared distance of 9 * sample - sum) is kept when centring on
 * it lowers their energy and grows their range by at most 12.5 %.  128
 * threads, one channel each, warp trees, then the four warps in order.
 * Returns the chosen sample (0..8) or -1. */
static int anchor_select(float samp[9][128], int64_t D) {
    enum { NS = 9, NT = 128 };
    float oe[NT], om[NT], cd[NS][NT];
    for (int t = 0; t < NT; ++t) {
        oe[t] = om[t] = 0.0f;
        for (int c = 0; c < NS; ++c) cd[c][t] = 0.0f;
        if (t >= D) continue;
        float sum = 0.0f;
        for (int s = 0; s < NS; ++s) {
            const float v = samp[s][t];
            oe[t] = fmaf(v, v, oe[t]);
            om[t] = fmaxf(om[t], fabsf(v));
            sum += v;
        }
        for (int c = 0; c < NS; ++c) {
            const float dist = fmaf(9.0f, samp[c][t], -sum);  /* 9 * x is exact */
            cd[c][t] = fmaf(dist, dist, cd[c][t]);
        }
    }
    float w_oe[4], w_om[4], w_cd[NS][4];
    for (int w = 0; w < 4; ++w) {
        w_oe[w] = warp_tree(oe + 32 * w, 0);
        w_om[w] = warp_tree(om + 32 * w, 1);
        for (int c = 0; c < NS; ++c) w_cd[c][w] = warp_tree(cd[c] + 32 * w, 0);
    }
    int best = 0;
    float best_d = 3.402823466e+38F;
    for (int c = 0; c < NS; ++c) {
        float d = 0.0f;
        for (int w = 0; w < 4; ++w) d += w_cd[c][w];
        if (d < best_d) {
            best = c;
            best_d = d;
        }
    }
    float be[NT], bm[NT];
    for (int t = 0; t < NT; ++t) {
        be[t] = bm[t] = 0.0f;
        if (t >= D) continue;
        for (int s = 0; s < NS; ++s) {
            const float r = samp[s][t] - samp[best][t];
            be[t] = fmaf(r, r, be[t]);
            bm[t] = fmaxf(bm[t], fabsf(r));
        }
    }
    float toe = 0.0f, tom = 0.0f, tbe = 0.0f, tbm = 0.0f;
    for (int w = 0; w < 4; ++w) {
        toe += w_oe[w];
        tom = fmaxf(tom, w_om[w]);
        tbe += warp_tree(be + 32 * w, 0);
        tbm = fmaxf(tbm, warp_tree(bm + 32 * w, 1));
    }
    return tbe < toe && tbm <= tom * 1.125f ? best : -1;
}

/* Anchor of the raw keys (DetectKAnchorKernel): nine rows s * (L - 1) / 8 of
 * K; anchor[o] = row index or -1, values[o, :] = that row as float or zeros
 * (values may be NULL). */
void orc_k_anchor(const uint16_t *k, int fp16, int64_t outer, int64_t L, int64_t D,
                  int64_t s_outer, int64_t s_tok, int32_t *anchor, float *values) {
    for (int64_t o = 0; o < outer; ++o) {
        float samp[9][128];
        for (int s = 0; s < 9; ++s) {
            const int64_t row = (int64_t)s * (L - 1) / 8;
            for (int c = 0; c < 128; ++c)
                samp[s][c] = c < D ? elem(k, o * s_outer + row * s_tok + c, fp16) : 0.0f;
        }
        const int sel = anchor_select(samp, D);
        anchor[o] = sel >= 0 ? (int32_t)((int64_t)sel * (L - 1) / 8) : -1;
        if (values)
            for (int64_t c = 0; c < D; ++c) values[o * D + c] = sel >= 0 ? samp[sel][c] : 0.0f;
    }
}

/* Anchor of the normalized + rotated keys of the fused prologue
 * (detect_anchor_kernel, qk_preprocess.cu:252-415): the nine sampled tokens
 * are processed as in process_row with their own RRMS (row scope: the row
 * RRMS; head scope: one FMA chain over channels 0..D-1, then the correctly
 * rounded 1/sqrt); the anchor's values are those processed floats.
 * k [B, H, L, D] contiguous bits; anchor [B, H]; values [B, H, D]. */
void orc_qk_anchor_processed(const uint16_t *k, const uint16_t *norm, const uint16_t *freqs,
                             int64_t B, int64_t H, int64_t L, int64_t D, int64_t fb, int64_t fs,
                             int rot_dim, int split_half, int row_scope, int fp16, float eps,
                             int32_t *anchor, float *values) {
    float nrm[128];
    for (int64_t b = 0; b < B; ++b)
        for (int64_t h = 0; h < H; ++h) {
            float samp[9][128];
            for (int s = 0; s < 9; ++s) {
                const int64_t tok = (int64_t)s * (L - 1) / 8;
                const uint16_t *row = k + ((b * H + h) * L + tok) * D;
                float rrms;
                if (row_scope) {
                    rrms = row_rrms(k, H, L, D, b, tok, fp16, eps);
                } else {
                    float sum = 0.0f;
                    for (int64_t c = 0; c < D; ++c) {
                        const float v = elem(row, c, fp16);
                        sum = fmaf(v, v, sum);
                    }
                    rrms = rsqrt_rn(sum / (float)D + eps);
                }
                for (int c = 0; c < 128; ++c) samp[s][c] = 0.0f;
                process_row(row, norm + (row_scope ? h * D : 0), freqs, b, tok, D, fb, fs,
                            rot_dim, split_half, fp16, rrms, nrm, samp[s]);
            }
            const int64_t o = b * H + h;
            const int sel = anchor_select(samp, D);
            anchor[o] = sel >= 0 ? (int32_t)((int64_t)sel * (L - 1) / 8) : -1;
            for (int64_t c = 0; c < D; ++c) values[o * D + c] = sel >= 0 ? samp[sel][c] : 0.0f;
        }
}

/* Randomized-Hadamard per-tile INT8 quantizer (quant_int8_tile, fused.cu:260-398;
 * quantize_tile, qk_preprocess.cu:417-563): per tile of T tokens (16: Q per
 * warp; 64: K per block) the rows, minus the anchor values [outer, D] when
 * given (K only; zeros = no anchor), are rotated (rot_row), amax starts at
 * 1e-7, scale = amax / 127, codes = rni(x * (127 / amax)) saturated, NaN ->
 * nan_code (0: cvt.rni.sat.s8 of fused.cu; -127: the prologue's
 * clamp(nearbyintf), qk_preprocess.cu:43-47).  IEEE divides (the reference's
 * extension uses --use_fast_math).  x and out share strides; scale is
 * [outer, tiles]. */
void orc_rot_quant(const uint16_t *x, int fp16, int64_t outer, int64_t L, int64_t D,
                   int64_t s_outer, int64_t s_tok, int64_t T, int64_t tiles,
                   const float *anchor_values, int nan_code, int8_t *out, float *scale) {
    float *buf = (float *)malloc(sizeof(float) * (size_t)(T * D));
    for (int64_t o = 0; o < outer; ++o) {
        const float *anc = anchor_values ? anchor_values + o * D : NULL;
        for (int64_t t = 0; t < tiles; ++t) {
            float amax = 0.0000001f;
            for (int64_t i = 0; i < T; ++i) {
                const int64_t tok = t * T + i;
                float *v = buf + i * D;
                if (tok >= L) continue;
                for (int64_t c = 0; c < D; ++c) {
                    v[c] = elem(x, o * s_outer + tok * s_tok + c, fp16);
                    if (anc) v[c] -= anc[c];
                }
                rot_row(v, (int)D);
                for (int64_t c = 0; c < D; ++c) amax = fmaxf(amax, fabsf(v[c]));
            }
            scale[o * tiles + t] = amax / 127.0f;
            const float inv = 127.0f / amax;
            for (int64_t i = 0; i < T; ++i) {
                const int64_t tok = t * T + i;
                if (tok >= L) continue;
                for (int64_t c = 0; c < D; ++c) {
                    const float y = buf[i * D + c] * inv;
                    out[o * s_outer + tok * s_tok + c] = isnan(y) ? (int8_t)nan_code : cvt_rni_sat_s8(y);
                }
            }
        }
    }
    free(buf);
}

/* Channel-wise INT8 V (quantize_value_kernel, quant_v_int8_cuda_sm75.cu:58-164):
 * per (outer, channel) amax over the L tokens, scale = max(amax / 127, 1e-12),
 * codes = rni_sat(v * (1 / scale)), written channel-major [outer, D, Lpad]
 * (tokens >= L zero).  The reference also permutes each run of 16 tokens for
 * its sm75 fragment loads; this layout is the un-permuted one. */
void orc_quant_v(const uint16_t *v, int fp16, int64_t outer, int64_t L, int64_t D,
                 int64_t s_outer, int64_t s_tok, int64_t Lpad, int8_t *codes, float *scale) {
    for (int64_t o = 0; o < outer; ++o) {
        for (int64_t c = 0; c < D; ++c) {
            float amax = 0.0f;
            for (int64_t t = 0; t < L; ++t)
                amax = fmaxf(amax, fabsf(elem(v, o * s_outer + t * s_tok + c, fp16)));
            const float sc = fmaxf(amax / 127.0f, 1.0e-12f);
            const float inv = 1.0f / sc;
            scale[o * D + c] = sc;
            int8_t *dst = codes + (o * D + c) * Lpad;
            for (int64_t t = 0; t < Lpad; ++t)
                dst[t] = t < L ? cvt_rni_sat_s8(elem(v, o * s_outer + t * s_tok + c, fp16) * inv) : 0;
        }
    }
}

/* cvt.rni.sat.u8.f32 (attn_utils.cuh:588-597). */
static inline int32_t cvt_rni_sat_u8(float x) {
    if (isnan(x)) return 0;
    float r = nearbyintf(x);
    if (r > 255.0f) r = 255.0f;
    if (r < 0.0f) r = 0.0f;
    return (int32_t)r;
}

/* Dense W8A8-PV attention (sparse_attention_kernel<UseW8A8, ForceDense>,
 * sol_sparse_cuda_sm75.cu:1197-1320; update_mdo / RS_to_u8 /
 * compute_int8_sv_permuted / normalize_d, attn_utils.cuh:465-585, 599-622,
 * 793-841, 923-965).  Per query row and 64-key block j, with
 * c_j = (sm_scale * log2 e) * q_scale[row / 16] * k_scale[j]:
 *   m_blk = fma(max_t s_t, c_j, -7.9943534)   (s_t = exact INT32 score;
 *           masked keys -5e6; 7.9943534 = log2 255)
 *   m' = max(m, m_blk);  d, O *= 2^(m - m');
 *   p_t = 2^fma(s_t, c_j, -m') in (0, 255];  P_t = rni_sat_u8(p_t)
 *         (masked keys: p_t = 0; the reference's -5e6 sentinel gives them
 *         2^fma(-5e6, c_j, -m'), which is exactly 0 in fp32 unless c_j is
 *         below ~2.6e-5, i.e. unless the Q/K scales are degenerate);
 *   d += sum p_t;  O[c] += (float)(sum_t P_t * V8[c, t])   (exact INT32)
 * and out[c] = O[c] * (1 / d) * v_scale[c] (fp32; the caller rounds to the
 * output dtype).  m starts at -5e6 and d at 1; exp2f stands for the
 * reference's ex2.approx.  q/k int8 [B, H, L, D] contiguous; v8 [B, Hk, D,
 * Lpad]; q_scale [B, Hq, q_tiles] (per 16 rows); k_scale [B, Hk, k_tiles]. */
void orc_w8a8_attn(const int8_t *q, const int8_t *k, const int8_t *v8, const float *v_scale,
                   const float *q_scale, const float *k_scale, int64_t B, int64_t Hq, int64_t Hk,
                   int64_t Lq, int64_t Lk, int64_t D, int64_t Lpad, int64_t q_tiles,
                   int64_t k_tiles, float sm_scale, int causal, float *out) {
    const float scale_log2 = sm_scale * 1.44269504088896340736f;
    const int64_t nblk = (Lk + 63) / 64;
    float *O = (float *)malloc(sizeof(float) * (size_t)D);
    for (int64_t b = 0; b < B; ++b) {
        for (int64_t h = 0; h < Hq; ++h) {
            const int64_t hk = h / (Hq / Hk);
            const int8_t *kh = k + (b * Hk + hk) * Lk * D;
            const int8_t *vh = v8 + (b * Hk + hk) * D * Lpad;
            const float *ksh = k_scale + (b * Hk + hk) * k_tiles;
            const float *vsh = v_scale + (b * Hk + hk) * D;
            for (int64_t i = 0; i < Lq; ++i) {
                const int8_t *qi = q + ((b * Hq + h) * Lq + i) * D;
                const float cq = scale_log2 * q_scale[(b * Hq + h) * q_tiles + i / 16];
                const int64_t nb = causal ? (i / 64 + 1 < nblk ? i / 64 + 1 : nblk) : nblk;
                float m = -5000000.0f, d = 1.0f;
                for (int64_t c = 0; c < D; ++c) O[c] = 0.0f;
                for (int64_t j = 0; j < nb; ++j) {
                    const float cj = cq * ksh[j];
                    float s[64];
                    float mx = -5000000.0f;
                    for (int t = 0; t < 64; ++t) {
                        const int64_t key = j * 64 + t;
                        if (key >= Lk || (causal && key > i)) {
                            s[t] = -5000000.0f;
                        } else {
                            int32_t acc = 0;
                            const int8_t *kk = kh + key * D;
                            for (int64_t c = 0; c < D; ++c) acc += (int32_t)qi[c] * (int32_t)kk[c];
                            s[t] = (float)acc;
                        }
                        mx = fmaxf(mx, s[t]);
                    }
                    const float m_new = fmaxf(m, fmaf(mx, cj, -7.9943534f));
                    const float f = exp2f(m - m_new);
                    d *= f;
                    for (int64_t c = 0; c < D; ++c) O[c] *= f;
                    m = m_new;
                    int32_t pu[64];
                    float psum = 0.0f;
                    for (int t = 0; t < 64; ++t) {
                        const int64_t key = j * 64 + t;
                        const int masked = key >= Lk || (causal && key > i);
                        const float pt = masked ? 0.0f : exp2f(fmaf(s[t], cj, -m));
                        pu[t] = cvt_rni_sat_u8(pt);
                        psum += pt;
                    }
                    d += psum;
                    for (int64_t c = 0; c < D; ++c) {
                        int32_t acc = 0;
                        const int8_t *vc = vh + c * Lpad + j * 64;
                        for (int t = 0; t < 64; ++t) acc += pu[t] * (int32_t)vc[t];
                        O[c] += (float)acc;
                    }
                }
                const float inv = 1.0f / d;
                float *orow = out + ((b * Hq + h) * Lq + i) * D;
                for (int64_t c = 0; c < D; ++c) orow[c] = O[c] * inv * vsh[c];
            }
        }
    }
    free(O);
}

/* ------------------------------------------------------------ helpers ---- */

void orc_f32_to_bf16(const float *x, int64_t n, uint16_t *out) {
    for (int64_t i = 0; i < n; ++i) out[i] = f32_to_bf16_rn(x[i]);
}

void orc_bf16_to_f32(const uint16_t *x, int64_t n, float *out) {
    for (int64_t i = 0; i < n; ++i) out[i] = bf16_to_f32(x[i]);
}

void orc_f32_to_f16(const float *x, int64_t n, uint16_t *out) {
    for (int64_t i = 0; i < n; ++i) out[i] = f32_to_f16_rn(x[i]);
}

void orc_f16_to_f32(const uint16_t *x, int64_t n, float *out) {
    for (int64_t i = 0; i < n; ++i) out[i] = f16_to_f32(x[i]);
}
