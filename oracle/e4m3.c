/*
 * CPU oracle for the FP8 (E4M3, "fn" flavour: no infinities, NaN = S.1111.111) byte arithmetic
 * of the KV store path.  TEST INFRASTRUCTURE ONLY: it is loaded by tests/, by
 * __graft_entry__.smoke() and by bench.py's cpu_baseline leg as the checker.  The product path
 * never links or calls it.
 *
 * What it restates:
 *   - nanovllm/layers/attention.py:27-31 (store_kvcache_kernel): `tl.store` of a bf16 value into a
 *     float8_e4m3fn pointer, i.e. an implicit bf16 -> e4m3 cast with round-to-nearest-even.  On the
 *     GPU Triton lowers that cast to the hardware `cvt.rn.satfinite` conversion, which saturates
 *     finite overflow to +-448 (mode E4M3_SATFINITE).  torch's `.to(torch.float8_e4m3fn)` is the
 *     same RNE rounding but maps |x| > 464 to NaN (mode E4M3_TORCH); both modes agree on every
 *     input with |x| <= 464.
 *   - nanovllm/kernels/fp8_attention.py:147-150,262-263,292-293: the e4m3 -> fp32 widening of
 *     cache bytes (no scale).
 *   - nanovllm/kernels/fp8_linear.py:24-28 (fp8_dyn_quant_kernel): the per-group quantiser
 *     convention scale = amax/448 (0 -> 1), clamp(x/scale, -448, 448), cast.  The reference
 *     applies it to GEMM activations; the store path's optional "scaled" mode applies it per
 *     (token, kv-head) row of head_dim values.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

enum { E4M3_SATFINITE = 0, E4M3_TORCH = 1 };

static float f32_from_bits(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static uint32_t bits_from_f32(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

float bf16_to_f32(uint16_t h) { return f32_from_bits(((uint32_t)h) << 16); }

/* fp32 -> e4m3fn byte, round to nearest, ties to even. */
uint8_t e4m3_from_f32(float x, int mode) {
    uint32_t u = bits_from_f32(x);
    uint8_t sign = (uint8_t)((u >> 24) & 0x80);
    float a = fabsf(x);
    if (isnan(x)) return (uint8_t)(mode == E4M3_TORCH ? (sign | 0x7F) : 0x7F);
    /* 464 is the midpoint between 448 (mantissa 110, even) and the unrepresentable 480; a tie
     * there rounds to 448, anything above rounds out of range. */
    if (a > 464.0f) {
        if (mode == E4M3_TORCH) return (uint8_t)(sign | 0x7F);
        return (uint8_t)(sign | 0x7E); /* satfinite: +-448 (also for +-inf) */
    }
    if (a == 0.0f) return sign;
    int e;
    frexpf(a, &e);          /* a = f * 2^e, f in [0.5, 1) -> floor(log2 a) = e - 1 */
    e -= 1;
    if (e < -6) {
        /* subnormal range: quantum 2^-9; q in [0, 8] (8 is the smallest normal, code 0x08) */
        float q = rintf(ldexpf(a, 9));
        return (uint8_t)(sign | (uint8_t)q);
    }
    float q = rintf(ldexpf(a, 3 - e)); /* in [8, 16] */
    int qi = (int)q;
    if (qi == 16) { qi = 8; e += 1; }
    int biased = e + 7;
    /* biased == 15 with mantissa 7 would be NaN; the a > 464 test above excludes it. */
    return (uint8_t)(sign | (uint8_t)(biased << 3) | (uint8_t)(qi - 8));
}

float e4m3_to_f32(uint8_t b) {
    int s = b >> 7, e = (b >> 3) & 0xF, m = b & 7;
    float v;
    if (e == 15 && m == 7) return NAN;
    if (e == 0) v = ldexpf((float)m, -9);
    else v = ldexpf((float)(8 + m), e - 10);
    return s ? -v : v;
}

/* Vector forms used through ctypes. */
void e4m3_from_bf16_vec(const uint16_t* in, uint8_t* out, int64_t n, int mode) {
    for (int64_t i = 0; i < n; ++i) out[i] = e4m3_from_f32(bf16_to_f32(in[i]), mode);
}

void e4m3_to_f32_vec(const uint8_t* in, float* out, int64_t n) {
    for (int64_t i = 0; i < n; ++i) out[i] = e4m3_to_f32(in[i]);
}

/* Scaled quantiser over rows of `d` bf16 values: scale = amax/448 (0 -> 1), bytes =
 * e4m3(clamp(x / scale, -448, 448)).  fminf/fmaxf return the non-NaN operand, as CUDA's do. */
void e4m3_quant_rows_bf16(const uint16_t* in, uint8_t* out, float* scales, int64_t rows, int d) {
    for (int64_t r = 0; r < rows; ++r) {
        const uint16_t* x = in + r * d;
        float amax = 0.0f;
        for (int i = 0; i < d; ++i) amax = fmaxf(amax, fabsf(bf16_to_f32(x[i])));
        float s = amax / 448.0f;
        if (!(s > 0.0f)) s = 1.0f;
        scales[r] = s;
        for (int i = 0; i < d; ++i) {
            float y = bf16_to_f32(x[i]) / s;
            y = fminf(fmaxf(y, -448.0f), 448.0f);
            out[r * d + i] = e4m3_from_f32(y, E4M3_SATFINITE);
        }
    }
}
