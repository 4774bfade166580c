/*
 * CPU restatement of the ltx-weights dequant + LoRA-merge path.
 *
 * TEST INFRASTRUCTURE ONLY: this file is the checker for the CUDA kernels in
 * ltx-rust_b200/csrc/dequant_merge.cu.  Only tests/, __graft_entry__.smoke()
 * and bench.py's CPU-baseline leg may load it.  The product library never
 * links or calls it.
 *
 * Parity: pinned by the reference's own golden vectors
 * (crates/ltx-weights/tests/fixtures/{fp8_e4m3fn_*,lora_parity_*}.safetensors,
 * copied into tests/golden/ by tests/golden/make_golden.py) and by the
 * known answers of crates/ltx-weights/src/fp8.rs:161-205 and
 * crates/ltx-weights/tests/integration.rs:400-587.
 *
 * Every rounding step follows the reference exactly:
 *   - FP8 decode is exact (crates/ltx-weights/src/fp8.rs:90-158).
 *   - scale:  v = fma(scale, v, +0.0)            (store.rs:505-507)
 *   - LoRA:   c = coeff * B[o][r]  (one rounding) (store.rs:786)
 *             w = fma(c, A[r][i], w), r ascending (store.rs:787-789)
 *   - deltas are applied in merge order           (store.rs:511-515)
 *   - bf16 output = round-to-nearest-even of the final f32 (half 2.7.1
 *     bf16::from_f32), NaN kept as a quiet NaN with its sign.
 * Compile with -ffp-contract=off so the compiler cannot fuse c*B into the FMA.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#include <pthread.h>
#include <stdlib.h>

enum { OR_F32 = 0, OR_F16 = 1, OR_BF16 = 2, OR_F8E4M3 = 3, OR_F8E5M2 = 4 };

static float bits_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static uint32_t f32_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

/* fp8.rs:90-120: S EEEE MMM, bias 7, 0x7F/0xFF NaN, no infinities. */
float oracle_decode_e4m3fn(uint8_t byte) {
    if (byte == 0x7F || byte == 0xFF) return NAN;
    uint32_t sign = (byte & 0x80) ? 0x80000000u : 0u;
    uint32_t e = (byte >> 3) & 0x0F, m = byte & 0x07;
    if (e == 0) {
        if (m == 0) return bits_f32(sign);
        /* subnormal: m * 2^-9, exact in f32 */
        return (sign ? -1.0f : 1.0f) * ldexpf((float)m, -9);
    }
    return bits_f32(sign | ((e + 120u) << 23) | (m << 20));
}

/* fp8.rs:127-158: S EEEEE MM, bias 15, IEEE inf/NaN. */
float oracle_decode_e5m2(uint8_t byte) {
    uint32_t sign = (byte & 0x80) ? 0x80000000u : 0u;
    uint32_t e = (byte >> 2) & 0x1F, m = byte & 0x03;
    if (e == 31) return m == 0 ? bits_f32(sign | 0x7F800000u) : NAN;
    if (e == 0) {
        if (m == 0) return bits_f32(sign);
        return (sign ? -1.0f : 1.0f) * ldexpf((float)m, -16);
    }
    return bits_f32(sign | ((e + 112u) << 23) | (m << 21));
}

float oracle_bf16_to_f32(uint16_t h) { return bits_f32((uint32_t)h << 16); }

/* IEEE binary16 -> binary32, exact (half::f16::to_f32). */
float oracle_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1F, m = h & 0x3FF;
    if (e == 31) return bits_f32(sign | 0x7F800000u | (m << 13));
    if (e == 0) {
        if (m == 0) return bits_f32(sign);
        return (sign ? -1.0f : 1.0f) * ldexpf((float)m, -24);
    }
    return bits_f32(sign | ((e + 112u) << 23) | (m << 13));
}

/* half 2.7.1 bf16::from_f32: RNE; NaN -> quiet NaN keeping sign and top bits. */
uint16_t oracle_f32_to_bf16(float f) {
    uint32_t x = f32_bits(f);
    if ((x & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((x >> 16) | 0x0040u);
    uint32_t round_bit = 0x00008000u;
    if ((x & round_bit) && (x & (3u * round_bit - 1u))) return (uint16_t)((x >> 16) + 1u);
    return (uint16_t)(x >> 16);
}

static float decode_elem(const void *base, int dtype, int64_t idx) {
    switch (dtype) {
    case OR_F32: return ((const float *)base)[idx];
    case OR_F16: return oracle_f16_to_f32(((const uint16_t *)base)[idx]);
    case OR_BF16: return oracle_bf16_to_f32(((const uint16_t *)base)[idx]);
    case OR_F8E4M3: return oracle_decode_e4m3fn(((const uint8_t *)base)[idx]);
    default: return oracle_decode_e5m2(((const uint8_t *)base)[idx]);
    }
}

/* One host thread's share of rows. */
typedef struct {
    const void *base; int base_dtype; int fp8_scaled; float scale;
    int64_t in, row0, row1;
    int n_deltas; const float *const *A; const float *const *B; const int *rank; const float *coeff;
    float *dst_f32; uint16_t *dst_bf16; float *row;
} read_job;

static void *read_rows(void *arg) {
    read_job *j = (read_job *)arg;
    const int64_t in = j->in;
    float *row = j->row;
    for (int64_t o = j->row0; o < j->row1; ++o) {
        for (int64_t i = 0; i < in; ++i) {
            float v = decode_elem(j->base, j->base_dtype, o * in + i);
            if (j->fp8_scaled) v = fmaf(j->scale, v, 0.0f);
            row[i] = v;
        }
        for (int d = 0; d < j->n_deltas; ++d) {
            const int R = j->rank[d];
            const float *brow = j->B[d] + o * R;
            for (int r = 0; r < R; ++r) {
                const float c = j->coeff[d] * brow[r];
                const float *arow = j->A[d] + (int64_t)r * in;
                for (int64_t i = 0; i < in; ++i) row[i] = fmaf(c, arow[i], row[i]);
            }
        }
        if (j->dst_f32) memcpy(j->dst_f32 + o * in, row, (size_t)in * sizeof(float));
        if (j->dst_bf16)
            for (int64_t i = 0; i < in; ++i) j->dst_bf16[o * in + i] = oracle_f32_to_bf16(row[i]);
    }
    return NULL;
}

/*
 * WeightStore::read for one [out, in] weight (store.rs:479-521).
 *   base:       raw bytes of the stored tensor (dtype `base_dtype`)
 *   has_scale:  an FP8 tensor with a sibling `{key}_scale` (store.rs:499-508)
 *   deltas:     n_deltas LowRankDelta factors, already decoded to f32
 *               (A[r][in], B[out][r], rank, coeff), applied in order.
 *   dst_f32:    [out*in] f32 result (may be NULL)
 *   dst_bf16:   [out*in] bf16 result (may be NULL)
 *   n_threads:  host threads; rows are split into contiguous blocks.
 * Returns 0, -1 on an unsupported dtype, -2 on an allocation failure.
 */
int oracle_read_weight(const void *base, int base_dtype, int has_scale, float scale,
                       int64_t out, int64_t in, int n_deltas, const float *const *A,
                       const float *const *B, const int *rank, const float *coeff,
                       float *dst_f32, uint16_t *dst_bf16, int n_threads) {
    if (base_dtype < OR_F32 || base_dtype > OR_F8E5M2) return -1;
    int fp8 = base_dtype == OR_F8E4M3 || base_dtype == OR_F8E5M2;
    if (n_threads < 1) n_threads = 1;
    if (n_threads > 256) n_threads = 256;
    if (out < n_threads) n_threads = out > 0 ? (int)out : 1;
    pthread_t tid[256];
    read_job jobs[256];
    float *rows = (float *)malloc((size_t)n_threads * (size_t)(in > 0 ? in : 1) * sizeof(float));
    if (!rows) return -2;
    int64_t per = (out + n_threads - 1) / n_threads;
    int launched[256];
    for (int t = 0; t < n_threads; ++t) {
        read_job *j = &jobs[t];
        j->base = base; j->base_dtype = base_dtype; j->fp8_scaled = fp8 && has_scale; j->scale = scale;
        j->in = in; j->row0 = t * per; j->row1 = (t + 1) * per < out ? (t + 1) * per : out;
        j->n_deltas = n_deltas; j->A = A; j->B = B; j->rank = rank; j->coeff = coeff;
        j->dst_f32 = dst_f32; j->dst_bf16 = dst_bf16; j->row = rows + (size_t)t * (size_t)in;
        launched[t] = 0;
    }
    /* threads 1..n-1 run concurrently; this thread takes block 0 (and any block
       whose thread could not be created) */
    for (int t = 1; t < n_threads; ++t)
        if (jobs[t].row0 < jobs[t].row1)
            launched[t] = pthread_create(&tid[t], NULL, read_rows, &jobs[t]) == 0;
    read_rows(&jobs[0]);
    for (int t = 1; t < n_threads; ++t) {
        if (launched[t]) pthread_join(tid[t], NULL);
        else if (jobs[t].row0 < jobs[t].row1) read_rows(&jobs[t]);
    }
    free(rows);
    return 0;
}

/* merge_lora coefficient (store.rs:606-615): strength.mul_add(alpha / rank, 0). */
float oracle_lora_coeff(float strength, float alpha, int rank) {
    return fmaf(strength, alpha / (float)rank, 0.0f);
}

/* IEEE f32 fused multiply-add (Rust f32::mul_add), for host-side schedule math. */
float oracle_fmaf(float a, float b, float c) { return fmaf(a, b, c); }

/* f32 exp as Rust's f32::exp (libm expf, correctly rounded in glibc). */
float oracle_expf(float x) { return expf(x); }

/* Blender::blend_with_pending (crates/ltx-chunk/src/blend.rs:284-298) over n
 * values: w_old = 1 - w_new, out = w_new.mul_add(new, w_old * old), f32 with
 * the two roundings of the reference (no contraction: -ffp-contract=off). */
void oracle_crossfade_blend(const float *old_v, const float *new_v, float w_new, long long n, float *out) {
    const float w_old = 1.0f - w_new;
    for (long long i = 0; i < n; ++i) {
        const float a = w_old * old_v[i];
        out[i] = fmaf(w_new, new_v[i], a);
    }
}
