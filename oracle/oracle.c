/*
 * CPU oracle for the B200 GEMM stack -- TEST INFRASTRUCTURE ONLY.
 *
 * Plain-C restatement of the reference study's checking algorithms, used by
 * tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg as the
 * checker. The product (libb200gemm.so and the b200gemm package) never links,
 * imports or calls anything here.
 *
 *   oracle_splitmix64 / oracle_pattern_vectors
 *       SplitMix64 finaliser and the 16-byte index pattern of
 *       src/memory/ldgsts.cu:226-246 (lo = mix(i), hi = mix(i ^ salt)).
 *       Pinned by SplitMix64's published first output for seed 0
 *       (mix(0x9E3779B97F4A7C15) = 0xE220A8397B1DCDAF).
 *   oracle_checksum_u32
 *       XOR and wrapping 64-bit sum of 32-bit words (the stream checksum).
 *   oracle_umma_reference
 *       reference_a / reference_b / reference_d of
 *       src/compute/umma_1sm.cu:577-586 and the global-row variant of
 *       src/compute/umma_2sm.cu:796-803: D[r][c] = depth * sum_k A[r,k] B[k,c].
 *   oracle_gemm_tn_f64 / oracle_gemm_tn_f32
 *       D = A * B^T for bf16 A (M x K) and B (N x K), row-major, accumulated
 *       in double (exact for the test sizes' purposes) or sequentially in
 *       float; the reference's oracle is the IEEE fp32 einsum "mkl,nkl->mnl"
 *       of src/gemm/gemm_comparison.py:2705-2722.
 *   oracle_bf16_round
 *       fp32 -> bf16 round-to-nearest-even on the bit pattern.
 */
#include <stdint.h>
#include <string.h>

#define PATTERN_SALT 0xD1B54A32D192ED03ULL

uint64_t oracle_splitmix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

/* out receives 4 uint32 words per 16-byte vector, vectors [start, start+count). */
void oracle_pattern_vectors(uint64_t start, int64_t count, uint32_t* out) {
    for (int64_t i = 0; i < count; ++i) {
        const uint64_t idx = start + (uint64_t)i;
        const uint64_t lo = oracle_splitmix64(idx);
        const uint64_t hi = oracle_splitmix64(idx ^ PATTERN_SALT);
        out[4 * i + 0] = (uint32_t)lo;
        out[4 * i + 1] = (uint32_t)(lo >> 32);
        out[4 * i + 2] = (uint32_t)hi;
        out[4 * i + 3] = (uint32_t)(hi >> 32);
    }
}

void oracle_checksum_u32(const uint32_t* words, int64_t n, uint32_t* xor_out, uint64_t* sum_out) {
    uint32_t x = 0;
    uint64_t s = 0;
    for (int64_t i = 0; i < n; ++i) {
        x ^= words[i];
        s += words[i];
    }
    *xor_out = x;
    *sum_out = s;
}

static int32_t ref_a(int row, int k) { return ((row + 3 * k) % 7) - 3; }
static int32_t ref_b(int k, int col) { return ((2 * k + col) % 5) - 2; }

/* D is (128*cta_group) x n, row-major. */
void oracle_umma_reference(int cta_group, int n, int depth, double* d) {
    const int m = 128 * cta_group;
    for (int r = 0; r < m; ++r) {
        for (int c = 0; c < n; ++c) {
            int64_t sum = 0;
            for (int k = 0; k < 16; ++k) sum += (int64_t)ref_a(r, k) * (int64_t)ref_b(k, c);
            d[(int64_t)r * n + c] = (double)depth * (double)sum;
        }
    }
}

static float bf16_to_f32(uint16_t h) {
    uint32_t bits = (uint32_t)h << 16;
    float f;
    memcpy(&f, &bits, sizeof(f));
    return f;
}

uint16_t oracle_bf16_round(float f) {
    uint32_t bits;
    memcpy(&bits, &f, sizeof(bits));
    if ((bits & 0x7F800000u) == 0x7F800000u && (bits & 0x007FFFFFu)) return (uint16_t)((bits >> 16) | 0x40);
    bits += 0x7FFFu + ((bits >> 16) & 1u);
    return (uint16_t)(bits >> 16);
}

void oracle_gemm_tn_f64(int64_t m, int64_t n, int64_t k, const uint16_t* a, const uint16_t* b,
                        double* d) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < m; ++i) {
        for (int64_t j = 0; j < n; ++j) {
            double acc = 0.0;
            const uint16_t* ar = a + i * k;
            const uint16_t* br = b + j * k;
            for (int64_t p = 0; p < k; ++p) acc += (double)bf16_to_f32(ar[p]) * (double)bf16_to_f32(br[p]);
            d[i * n + j] = acc;
        }
    }
}

void oracle_gemm_tn_f32(int64_t m, int64_t n, int64_t k, const uint16_t* a, const uint16_t* b,
                        float* d) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < m; ++i) {
        for (int64_t j = 0; j < n; ++j) {
            float acc = 0.0f;
            const uint16_t* ar = a + i * k;
            const uint16_t* br = b + j * k;
            for (int64_t p = 0; p < k; ++p) acc += bf16_to_f32(ar[p]) * bf16_to_f32(br[p]);
            d[i * n + j] = acc;
        }
    }
}
