/*
 * gk_common.h - definitions shared by the CUDA kernels and the CPU oracle.
 *
 * Everything here is plain C99 that also compiles as CUDA __host__ __device__
 * code, so the GPU path and the CPU oracle use the same constants, the same
 * random streams and the same injected evaluator, bit for bit.
 *
 * Contents
 *   - the int32 [N,170] state wire record (python/kingdom_ai/gpu_rules.py:16-33)
 *   - the 96-bit padded bitboard used by the kernels (rows of 10 bits, the
 *     10th column is always zero, so +-1 shifts need no column mask)
 *   - PCG32 (O'Neill 2014, "PCG: A Family of Simple Fast Space-Efficient
 *     Statistically Good Algorithms for Random Number Generation",
 *     pcg32_srandom_r / pcg32_random_r, XSH-RR 64/32) and the bounded draw
 *     floor(r * n / 2^32) used by the playout and position generators
 *   - SplitMix64 (Steele, Lea, Flood 2014) used by the injected evaluator
 *   - gk_exp_det: a deterministic exp built only from IEEE-754 double
 *     add/sub/mul (Cody-Waite range reduction by ln 2 and a degree-13 Taylor
 *     polynomial in Horner form) so that host and device produce identical
 *     bits. Device code uses __dadd_rn/__dmul_rn so nvcc cannot contract into
 *     FMA; host code must be compiled with -ffp-contract=off.
 */
#ifndef GK_COMMON_H
#define GK_COMMON_H

#include <stdint.h>

#if defined(__CUDACC__)
#define GK_HD __host__ __device__ __forceinline__
#else
#define GK_HD static inline
#endif

/* ----------------------------------------------------------------------- */
/* Wire record: python/kingdom_ai/gpu_rules.py:16-33                       */
/* ----------------------------------------------------------------------- */
#define GK_STATE_WIDTH 170
#define GK_CELLS 81
#define GK_ACTIONS 82
#define GK_PASS 81
#define GK_ACTOR 162
#define GK_BLACK_STOCK 163
#define GK_WHITE_STOCK 164
#define GK_PASSES 165
#define GK_REASON 166
#define GK_WINNER 167
#define GK_CAPTURED 168
#define GK_RESERVED 169
/* GPU wire end-reason codes (differ from C++ EndReason order). */
#define GK_NONE 0
#define GK_CAPTURE 1
#define GK_SUICIDE 2
#define GK_TWO_PASSES 3
/* C++ kingdom::EndReason order (engine/include/board/GameResult.h:7). */
#define GK_CPP_NONE 0
#define GK_CPP_CAPTURE 1
#define GK_CPP_TWO_PASSES 2
#define GK_CPP_SUICIDE 3
#define GK_STONES 41
#define GK_PLANES 10
#define GK_FEATURES (GK_PLANES * GK_CELLS)
/* Longest possible game: every placement and pass alternate (gpu_training.py:24). */
#define GK_MAX_PLIES (2 * GK_CELLS + 2)

/* Error bits shared by every entry point and kernel status word. */
#define GK_ERR_CAPACITY 1u   /* tree capacity exhausted or illegal stored edge */
#define GK_ERR_BAD_EVAL 2u   /* non-finite policy/value or value outside [-1,1] */
#define GK_ERR_TIMEOUT 4u    /* a bounded device-side wait gave up */
#define GK_ERR_BAD_INPUT 8u  /* a record outside the wire format's value ranges */

/* ----------------------------------------------------------------------- */
/* Bitboards: cell (r, c) -> bit r*10 + c of a 96-bit little-endian value    */
/* ----------------------------------------------------------------------- */
typedef struct {
    uint32_t w[3];
} gk_b96;

/* Packed device state: 16 x u32 = 64 bytes.
 *   w[0..2] black stones    w[3..5] white stones   w[6..8] neutral stones
 *   w[9..11] black-owned    w[12..14] white-owned  w[15] scalar fields      */
typedef struct {
    uint32_t w[16];
} gk_bits;

#define GK_META_ACTOR_SHIFT 0     /* 2 bits: 1 black, 2 white */
#define GK_META_BSTOCK_SHIFT 2    /* 6 bits: 0..41 */
#define GK_META_WSTOCK_SHIFT 8    /* 6 bits */
#define GK_META_PASSES_SHIFT 14   /* 2 bits: 0..2 */
#define GK_META_REASON_SHIFT 16   /* 2 bits: wire reason code */
#define GK_META_WINNER_SHIFT 18   /* 2 bits: 0, 1, 2 */
#define GK_META_CAPTURED_SHIFT 20 /* 7 bits: 0..81 */
/* Bit 27: territory settled. Set only by the device transitions (initial state
 * and every placement, which run the territory claim) and meaning that every
 * empty component that qualifies as territory is already owned; states packed
 * from wire records have it clear, and their next placement runs the full
 * claim over the whole board. A state settled this way needs only the
 * component the new stone splits to be re-examined. Bits 28..31 are zero. */
#define GK_META_SETTLED (1u << 27)

#define GK_VALID0 0xdff7fdffu
#define GK_VALID1 0xf7fdff7fu
#define GK_VALID2 0x01ff7fdfu
#define GK_ROW0_0 0x000001ffu
#define GK_ROW8_2 0x01ff0000u
#define GK_COL0_0 0x40100401u
#define GK_COL0_1 0x10040100u
#define GK_COL0_2 0x00010040u
#define GK_COL8_0 0x10040100u
#define GK_COL8_1 0x04010040u
#define GK_COL8_2 0x01004010u

GK_HD int gk_cell_bit(int cell) { return cell + cell / 9; }
GK_HD int gk_bit_cell(int bit) { return bit - bit / 10; }

GK_HD gk_b96 gk_b(uint32_t a, uint32_t b, uint32_t c) {
    gk_b96 r;
    r.w[0] = a; r.w[1] = b; r.w[2] = c;
    return r;
}
GK_HD gk_b96 gk_valid(void) { return gk_b(GK_VALID0, GK_VALID1, GK_VALID2); }
GK_HD gk_b96 gk_or(gk_b96 a, gk_b96 b) { return gk_b(a.w[0] | b.w[0], a.w[1] | b.w[1], a.w[2] | b.w[2]); }
GK_HD gk_b96 gk_and(gk_b96 a, gk_b96 b) { return gk_b(a.w[0] & b.w[0], a.w[1] & b.w[1], a.w[2] & b.w[2]); }
GK_HD gk_b96 gk_andnot(gk_b96 a, gk_b96 b) { return gk_b(a.w[0] & ~b.w[0], a.w[1] & ~b.w[1], a.w[2] & ~b.w[2]); }
GK_HD int gk_any(gk_b96 a) { return (a.w[0] | a.w[1] | a.w[2]) != 0u; }
GK_HD int gk_eq(gk_b96 a, gk_b96 b) {
    return ((a.w[0] ^ b.w[0]) | (a.w[1] ^ b.w[1]) | (a.w[2] ^ b.w[2])) == 0u;
}
GK_HD gk_b96 gk_single(int bit) {
    gk_b96 r = gk_b(0u, 0u, 0u);
    r.w[bit >> 5] = 1u << (bit & 31);
    return r;
}
GK_HD int gk_test(gk_b96 a, int bit) { return (int)((a.w[bit >> 5] >> (bit & 31)) & 1u); }

GK_HD int gk_popc32(uint32_t v) {
#if defined(__CUDA_ARCH__)
    return __popc(v);
#else
    return __builtin_popcount(v);
#endif
}
GK_HD int gk_popc(gk_b96 a) { return gk_popc32(a.w[0]) + gk_popc32(a.w[1]) + gk_popc32(a.w[2]); }

/* 96-bit shifts by s in 1..31 (funnel shifts on the device). */
GK_HD gk_b96 gk_shl(gk_b96 a, int s) {
    gk_b96 r;
#if defined(__CUDA_ARCH__)
    r.w[2] = __funnelshift_l(a.w[1], a.w[2], s);
    r.w[1] = __funnelshift_l(a.w[0], a.w[1], s);
#else
    r.w[2] = (a.w[2] << s) | (a.w[1] >> (32 - s));
    r.w[1] = (a.w[1] << s) | (a.w[0] >> (32 - s));
#endif
    r.w[0] = a.w[0] << s;
    return r;
}
GK_HD gk_b96 gk_shr(gk_b96 a, int s) {
    gk_b96 r;
#if defined(__CUDA_ARCH__)
    r.w[0] = __funnelshift_r(a.w[0], a.w[1], s);
    r.w[1] = __funnelshift_r(a.w[1], a.w[2], s);
#else
    r.w[0] = (a.w[0] >> s) | (a.w[1] << (32 - s));
    r.w[1] = (a.w[1] >> s) | (a.w[2] << (32 - s));
#endif
    r.w[2] = a.w[2] >> s;
    return r;
}
/* Orthogonal neighbours of a set (not including the set), clipped to the board. */
GK_HD gk_b96 gk_neighbours(gk_b96 a) {
    gk_b96 r = gk_or(gk_or(gk_shl(a, 1), gk_shr(a, 1)), gk_or(gk_shl(a, 10), gk_shr(a, 10)));
    return gk_and(r, gk_valid());
}
/* Connected closure of `seed` inside `mask` (4-connectivity). */
GK_HD gk_b96 gk_flood(gk_b96 mask, gk_b96 seed) {
    gk_b96 x = gk_and(seed, mask);
    for (;;) {
        gk_b96 y = gk_and(gk_or(x, gk_or(gk_or(gk_shl(x, 1), gk_shr(x, 1)),
                                         gk_or(gk_shl(x, 10), gk_shr(x, 10)))), mask);
        if (gk_eq(x, y)) return x;
        x = y;
    }
}

GK_HD gk_b96 gk_get(const gk_bits* s, int plane) {
    return gk_b(s->w[3 * plane], s->w[3 * plane + 1], s->w[3 * plane + 2]);
}
GK_HD void gk_put(gk_bits* s, int plane, gk_b96 v) {
    s->w[3 * plane] = v.w[0]; s->w[3 * plane + 1] = v.w[1]; s->w[3 * plane + 2] = v.w[2];
}
#define GK_PLANE_BLACK 0
#define GK_PLANE_WHITE 1
#define GK_PLANE_NEUTRAL 2
#define GK_PLANE_OWN_BLACK 3
#define GK_PLANE_OWN_WHITE 4

GK_HD int gk_meta(const gk_bits* s, int shift, uint32_t mask) { return (int)((s->w[15] >> shift) & mask); }
GK_HD int gk_actor(const gk_bits* s) { return gk_meta(s, GK_META_ACTOR_SHIFT, 3u); }
GK_HD int gk_reason(const gk_bits* s) { return gk_meta(s, GK_META_REASON_SHIFT, 3u); }
GK_HD int gk_winner(const gk_bits* s) { return gk_meta(s, GK_META_WINNER_SHIFT, 3u); }
GK_HD int gk_passes(const gk_bits* s) { return gk_meta(s, GK_META_PASSES_SHIFT, 3u); }
GK_HD int gk_stock(const gk_bits* s, int player) {
    return player == 1 ? gk_meta(s, GK_META_BSTOCK_SHIFT, 63u) : gk_meta(s, GK_META_WSTOCK_SHIFT, 63u);
}
GK_HD int gk_captured(const gk_bits* s) { return gk_meta(s, GK_META_CAPTURED_SHIFT, 127u); }
GK_HD uint32_t gk_pack_meta(int actor, int bstock, int wstock, int passes, int reason, int winner,
                            int captured) {
    return ((uint32_t)actor << GK_META_ACTOR_SHIFT) | ((uint32_t)bstock << GK_META_BSTOCK_SHIFT) |
           ((uint32_t)wstock << GK_META_WSTOCK_SHIFT) | ((uint32_t)passes << GK_META_PASSES_SHIFT) |
           ((uint32_t)reason << GK_META_REASON_SHIFT) | ((uint32_t)winner << GK_META_WINNER_SHIFT) |
           ((uint32_t)captured << GK_META_CAPTURED_SHIFT);
}

/* ----------------------------------------------------------------------- */
/* PCG32 (XSH-RR 64/32), O'Neill 2014                                       */
/* ----------------------------------------------------------------------- */
typedef struct {
    uint64_t state;
    uint64_t inc;
} gk_pcg32;

GK_HD uint32_t gk_pcg32_next(gk_pcg32* rng) {
    uint64_t old = rng->state;
    rng->state = old * 6364136223846793005ULL + rng->inc;
    uint32_t xorshifted = (uint32_t)(((old >> 18u) ^ old) >> 27u);
    uint32_t rot = (uint32_t)(old >> 59u);
    return (xorshifted >> rot) | (xorshifted << ((0u - rot) & 31u));
}
/* pcg32_srandom_r(initstate = seed, initseq = stream). */
GK_HD gk_pcg32 gk_pcg32_seed(uint64_t seed, uint64_t stream) {
    gk_pcg32 rng;
    rng.state = 0u;
    rng.inc = (stream << 1u) | 1u;
    (void)gk_pcg32_next(&rng);
    rng.state += seed;
    (void)gk_pcg32_next(&rng);
    return rng;
}
/* Uniform index in [0, n): floor(r * n / 2^32) (multiply-shift, no rejection). */
GK_HD uint32_t gk_pcg32_bounded(gk_pcg32* rng, uint32_t n) {
    return (uint32_t)(((uint64_t)gk_pcg32_next(rng) * (uint64_t)n) >> 32u);
}

/* ----------------------------------------------------------------------- */
/* SplitMix64 finaliser                                                     */
/* ----------------------------------------------------------------------- */
GK_HD uint64_t gk_splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ULL;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

/* ----------------------------------------------------------------------- */
/* Deterministic double arithmetic                                          */
/* ----------------------------------------------------------------------- */
#if defined(__CUDA_ARCH__)
#define GK_DADD(a, b) __dadd_rn((a), (b))
#define GK_DSUB(a, b) __dadd_rn((a), -(b))
#define GK_DMUL(a, b) __dmul_rn((a), (b))
#else
#define GK_DADD(a, b) ((a) + (b))
#define GK_DSUB(a, b) ((a) - (b))
#define GK_DMUL(a, b) ((a) * (b))
#endif

GK_HD double gk_pow2i(int k) {
    /* 2^k for k in [-1022, 1023], built from the exponent bits (exact). */
    union {
        uint64_t u;
        double d;
    } v;
    v.u = (uint64_t)(k + 1023) << 52;
    return v.d;
}

/* exp(x) for |x| <= 700 from IEEE double add/sub/mul only.
 * Cody-Waite: k = round(x / ln2), r = (x - k*LN2_HI) - k*LN2_LO with LN2_HI
 * holding the leading 32 bits of ln 2 (so k*LN2_HI is exact for |k| < 2^20),
 * |r| <= 0.3466; then exp(r) by its Taylor series to degree 13 (truncation
 * error below 2e-17 relative) in Horner form, scaled by 2^k. */
GK_HD double gk_exp_det(double x) {
    const double LOG2E = 1.4426950408889634;
    const double LN2_HI = 6.93147180369123816490e-01; /* 0x3FE62E42FEE00000 */
    const double LN2_LO = 1.90821492927058770002e-10; /* ln2 - LN2_HI */
    double t = GK_DADD(GK_DMUL(x, LOG2E), 0.5);
    double kf = (double)(int64_t)t;
    if (kf > t) kf = GK_DSUB(kf, 1.0); /* floor for negative t */
    int k = (int)kf;
    double r = GK_DSUB(GK_DSUB(x, GK_DMUL(kf, LN2_HI)), GK_DMUL(kf, LN2_LO));
    double p = 1.0 / 6227020800.0;                 /* 1/13! */
    p = GK_DADD(GK_DMUL(p, r), 1.0 / 479001600.0); /* 1/12! */
    p = GK_DADD(GK_DMUL(p, r), 1.0 / 39916800.0);  /* 1/11! */
    p = GK_DADD(GK_DMUL(p, r), 1.0 / 3628800.0);   /* 1/10! */
    p = GK_DADD(GK_DMUL(p, r), 1.0 / 362880.0);    /* 1/9!  */
    p = GK_DADD(GK_DMUL(p, r), 1.0 / 40320.0);     /* 1/8!  */
    p = GK_DADD(GK_DMUL(p, r), 1.0 / 5040.0);      /* 1/7!  */
    p = GK_DADD(GK_DMUL(p, r), 1.0 / 720.0);       /* 1/6!  */
    p = GK_DADD(GK_DMUL(p, r), 1.0 / 120.0);       /* 1/5!  */
    p = GK_DADD(GK_DMUL(p, r), 1.0 / 24.0);        /* 1/4!  */
    p = GK_DADD(GK_DMUL(p, r), 1.0 / 6.0);         /* 1/3!  */
    p = GK_DADD(GK_DMUL(p, r), 0.5);               /* 1/2!  */
    p = GK_DADD(GK_DMUL(p, r), 1.0);               /* 1/1!  */
    p = GK_DADD(GK_DMUL(p, r), 1.0);               /* 1/0!  */
    return GK_DMUL(p, gk_pow2i(k));
}

/* ----------------------------------------------------------------------- */
/* Injected evaluator for the fixed-evaluator PUCT workload                 */
/* ----------------------------------------------------------------------- */
/* A pure function of the canonical wire record. The record is packed into
 * 7 words (2-bit cell codes, 2-bit owner codes, one scalar word) and chained
 * through SplitMix64. Each action's logit z_a is an Irwin-Hall(4) variate
 * (four 16-bit uniforms) rescaled to unit variance, an approximately N(0,1)
 * draw; its weight is w_a = exp(z_a) rounded to float, so the expansion's
 * (w / max) / sum normalisation is the softmax of the logits. The value is a
 * uniform draw in [-1, 1) rounded to float. Weights are produced for all 82
 * actions; the search masks illegal ones. */
#define GK_EVAL_WORDS 7

GK_HD uint64_t gk_eval_hash_words(const uint64_t* words) {
    uint64_t h = 0x243F6A8885A308D3ULL;
    for (int i = 0; i < GK_EVAL_WORDS; ++i) h = gk_splitmix64(h ^ words[i]);
    return h;
}

GK_HD float gk_eval_weight(uint64_t h, int action) {
    uint64_t u = gk_splitmix64(h + (uint64_t)(action + 1) * 0xD1B54A32D192ED03ULL);
    uint32_t s = (uint32_t)(u & 0xFFFFu) + (uint32_t)((u >> 16) & 0xFFFFu) +
                 (uint32_t)((u >> 32) & 0xFFFFu) + (uint32_t)((u >> 48) & 0xFFFFu);
    /* s / 65536 is an exact double in [0, 4); mean 2, variance 1/3. */
    double z = GK_DMUL(GK_DSUB(GK_DMUL((double)s, 1.0 / 65536.0), 2.0), 1.7320508075688772);
    return (float)gk_exp_det(z);
}

GK_HD float gk_eval_value(uint64_t h) {
    uint64_t u = gk_splitmix64(h ^ 0x8CB92BA72F3D8DD7ULL);
    double unit = GK_DMUL((double)(u >> 11), 1.0 / 9007199254740992.0); /* [0, 1) */
    return (float)GK_DSUB(GK_DMUL(unit, 2.0), 1.0);
}

/* Pack a wire record (int32[170]) into the evaluator's 7 words. */
GK_HD void gk_eval_words_from_record(const int32_t* rec, uint64_t* words) {
    for (int i = 0; i < GK_EVAL_WORDS; ++i) words[i] = 0u;
    for (int i = 0; i < GK_CELLS; ++i) {
        words[i >> 5] |= (uint64_t)(rec[i] & 3) << (2 * (i & 31));
        words[3 + (i >> 5)] |= (uint64_t)(rec[GK_CELLS + i] & 3) << (2 * (i & 31));
    }
    words[6] = (uint64_t)(uint32_t)rec[GK_ACTOR] | ((uint64_t)(uint32_t)rec[GK_BLACK_STOCK] << 8) |
               ((uint64_t)(uint32_t)rec[GK_WHITE_STOCK] << 16) |
               ((uint64_t)(uint32_t)rec[GK_PASSES] << 24) |
               ((uint64_t)(uint32_t)rec[GK_REASON] << 32) |
               ((uint64_t)(uint32_t)rec[GK_WINNER] << 40) |
               ((uint64_t)(uint32_t)rec[GK_CAPTURED] << 48);
}

/* Cells 9r+c of a 96-bit board (rows of 10 bits) as an 81-bit mask:
 * *lo holds cells 0..63, *hi cells 64..80. */
GK_HD void gk_board_cells(gk_b96 b, uint64_t* lo, uint64_t* hi) {
    const uint64_t blo = (uint64_t)b.w[0] | ((uint64_t)b.w[1] << 32), bhi = b.w[2];
    uint64_t l = 0u, h = 0u;
    for (int r = 0; r < 9; ++r) {
        const int src = 10 * r, dst = 9 * r;
        uint64_t row;
        if (src + 9 <= 64) row = (blo >> src) & 0x1FFu;
        else if (src >= 64) row = (bhi >> (src - 64)) & 0x1FFu;
        else row = ((blo >> src) | (bhi << (64 - src))) & 0x1FFu;
        if (dst + 9 <= 64) l |= row << dst;
        else if (dst >= 64) h |= row << (dst - 64);
        else {
            l |= row << dst;
            h |= row >> (64 - dst);
        }
    }
    *lo = l;
    *hi = h;
}

/* Bit j of the low 32 bits of x -> bit 2j. */
GK_HD uint64_t gk_spread32(uint64_t x) {
    x &= 0xFFFFFFFFull;
    x = (x | (x << 16)) & 0x0000FFFF0000FFFFull;
    x = (x | (x << 8)) & 0x00FF00FF00FF00FFull;
    x = (x | (x << 4)) & 0x0F0F0F0F0F0F0F0Full;
    x = (x | (x << 2)) & 0x3333333333333333ull;
    x = (x | (x << 1)) & 0x5555555555555555ull;
    return x;
}

/* Same 7 words computed directly from the packed bitboard state: the 2-bit
 * codes of gk_eval_words_from_record (cell: black 1, else white 2, else
 * neutral 3; owner: black 1, else white 2) as two bit-planes each, compacted
 * to cell order and interleaved. */
GK_HD void gk_eval_words_from_bits(const gk_bits* s, uint64_t* words) {
    const gk_b96 black = gk_get(s, GK_PLANE_BLACK), white = gk_get(s, GK_PLANE_WHITE);
    const gk_b96 neutral = gk_get(s, GK_PLANE_NEUTRAL);
    const gk_b96 ob = gk_get(s, GK_PLANE_OWN_BLACK), ow = gk_get(s, GK_PLANE_OWN_WHITE);
    gk_b96 planes[4];
    planes[0] = gk_or(black, gk_andnot(neutral, white));       /* cell code bit 0 */
    planes[1] = gk_andnot(gk_or(white, neutral), black);       /* cell code bit 1 */
    planes[2] = ob;                                            /* owner code bit 0 */
    planes[3] = gk_andnot(ow, ob);                             /* owner code bit 1 */
    for (int k = 0; k < 2; ++k) {
        uint64_t lo0, hi0, lo1, hi1;
        gk_board_cells(planes[2 * k], &lo0, &hi0);
        gk_board_cells(planes[2 * k + 1], &lo1, &hi1);
        words[3 * k] = gk_spread32(lo0) | (gk_spread32(lo1) << 1);
        words[3 * k + 1] = gk_spread32(lo0 >> 32) | (gk_spread32(lo1 >> 32) << 1);
        words[3 * k + 2] = gk_spread32(hi0) | (gk_spread32(hi1) << 1);
    }
    words[6] = (uint64_t)gk_actor(s) | ((uint64_t)gk_stock(s, 1) << 8) | ((uint64_t)gk_stock(s, 2) << 16) |
               ((uint64_t)gk_passes(s) << 24) | ((uint64_t)gk_reason(s) << 32) |
               ((uint64_t)gk_winner(s) << 40) | ((uint64_t)gk_captured(s) << 48);
}

#endif /* GK_COMMON_H */
