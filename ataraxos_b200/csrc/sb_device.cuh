// sb_device.cuh -- device-side building blocks of the B200 Stratego simulator.
//
// One warp owns one env at a time.  The env's 256-byte record is staged in
// shared memory, the 100 squares are spread over the 32 lanes (square
// lane + 32k), and everything that is per-env scalar (validating and applying
// the action, the trackers) runs warp-uniformly: every lane computes the same
// values from shared memory and lane 0 stores them.
//
// Board square code (1 byte per square, packed 10x10):
//   bits 0-3 piece type (0 none, 1 Spy .. 10 Marshal, 11 Flag, 12 Bomb)
//   bit  4   owner is Blue (only meaningful when bit 5 is set)
//   bit  5   occupied
//   bit  6   moved flag of the square   (csrc/stratego_buffer.cu:243-253)
//   bit  7   revealed flag of the square
// Empty squares keep bits 0-5 clear; bits 6-7 are per-square tracker flags
// that survive the piece leaving, as in the reference's bool[100] tensors.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace sb {

constexpr int NSQ = 100;
constexpr int NACT = 10000;
constexpr int NHIST = 32;
constexpr int NRING = 64;
constexpr int NCH = 488;
constexpr int REC = 256;
constexpr unsigned FULL = 0xffffffffu;

// Record layout (byte offsets).  Every field is naturally aligned.
constexpr int R_BOARD = 0;      // u8[100]
constexpr int R_PLAYER = 100;   // i8  side to move (0 Red, 1 Blue)
constexpr int R_OUTCOME = 101;  // i8  -1 ongoing, 0 red win, 1 blue win, 2 draw
constexpr int R_TERM = 102;     // u8
constexpr int R_FLAGCAP = 103;  // u8
constexpr int R_MOVENUM = 104;  // i32
constexpr int R_MSA = 108;      // i32 moves since last attack
constexpr int R_TSINCE = 112;   // i32 terminated_since
constexpr int R_HHEAD = 116;    // u8  history ring head
constexpr int R_HLEN = 117;     // u8  history ring length
constexpr int R_TSVIOL = 118;   // u8  two-square violation (sticky)
constexpr int R_CHVIOL = 119;   // u8  chasing violation (sticky)
constexpr int R_TSCOUNT = 120;  // i32[2]
constexpr int R_TSLO = 128;     // i16[2]
constexpr int R_TSHI = 132;     // i16[2]
constexpr int R_CHHEAD = 136;   // u8[2]
constexpr int R_CHLEN = 138;    // u8[2]
constexpr int R_CHLAST = 140;   // i8[2]
constexpr int R_PROP = 142;     // i16 cached proposal (-1 none)
constexpr int R_ZHASH = 144;    // i64 Zobrist hash of the board
constexpr int R_EPISODE = 152;  // i32 pool resets done in this env
constexpr int R_INVALID = 156;  // i32 rejected actions
constexpr int R_PROPPLY = 160;  // i32 ply the cached proposal was drawn for (-1 stale)
constexpr int R_NLEGAL = 164;   // i16 legal moves of the side to move (with the proposal)
constexpr int R_PROPKIND = 166; // u8  policy the cached proposal was drawn with
constexpr int R_PROPLP = 168;   // f32 log-prob of the cached proposal
constexpr int R_HIST = 176;     // i16[32] move-history ring
constexpr int R_BLOOM = 240;    // u64[2] per-side Bloom filter of the chase ring's hashes
// Under the ISF repetition rules the per-mover two-square fields (120-135)
// are unused and these take their bytes:
constexpr int R_ISF_THR = 120;  // i8[2][4] squares each side's last move threatened (-1 none)
constexpr int R_ISF_EV = 128;   // u8  bit p: side p's last move was an evasion
constexpr int ISF_TS_BYTES = 600;  // per env: 100 squares x (lo,hi) x 3 segment intersections

constexpr uint8_t C_PIECE = 15, C_BLUE = 16, C_OCC = 32, C_MOVED = 64, C_REV = 128;

enum : uint32_t {
    TAG_SETUP = 1,
    TAG_RESET = 2,
    TAG_ACTION = 3,
    TAG_LOGIT = 4,
    TAG_BELIEF = 6,
};

template <typename T>
__device__ __forceinline__ T& fld(uint8_t* rec, int off) {
    return *reinterpret_cast<T*>(rec + off);
}
template <typename T>
__device__ __forceinline__ const T& fld(const uint8_t* rec, int off) {
    return *reinterpret_cast<const T*>(rec + off);
}

// Lakes: rows 4-5, columns 2, 3, 6, 7 (stratego/constants.py:25-28).
__device__ __forceinline__ bool is_lake(int sq) {
    return sq >= 40 && sq < 60 && ((0xCCu >> (sq % 10)) & 1u);
}
__device__ __forceinline__ bool can_move(int pt) { return pt >= 1 && pt <= 10; }
__device__ __forceinline__ int owner_of(uint8_t c) { return (c & C_OCC) ? ((c >> 4) & 1) : -1; }

// Zobrist entry [sq][owner][piece] of a [10,10,2,13] table (global or shared).
__device__ __forceinline__ uint64_t zob(const int64_t* z, int sq, int owner, int piece) {
    return (uint64_t)z[(sq * 2 + owner) * 13 + piece];
}

// Philox4x32-10 (Salmon, Moraes, Dror, Shaw, SC'11).
__device__ __forceinline__ uint4 philox(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3, uint64_t seed) {
    uint32_t k0 = (uint32_t)seed, k1 = (uint32_t)(seed >> 32);
#pragma unroll
    for (int r = 0; r < 10; ++r) {
        uint32_t hi0 = __umulhi(0xD2511F53u, c0), lo0 = 0xD2511F53u * c0;
        uint32_t hi1 = __umulhi(0xCD9E8D57u, c2), lo1 = 0xCD9E8D57u * c2;
        uint32_t n0 = hi1 ^ c1 ^ k0, n2 = hi0 ^ c3 ^ k1;
        c0 = n0; c1 = lo1; c2 = n2; c3 = lo0;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    return make_uint4(c0, c1, c2, c3);
}

// The same generator with its ten round keys precomputed (rk[2r], rk[2r+1] =
// the key halves after r bumps): kernels read them from their parameter block,
// so each round's key enters the XOR as an operand instead of being bumped
// with two additions.
__host__ __device__ __forceinline__ void philox_round_keys(uint64_t seed, uint32_t rk[20]) {
    uint32_t k0 = (uint32_t)seed, k1 = (uint32_t)(seed >> 32);
    for (int r = 0; r < 10; ++r) {
        rk[2 * r] = k0;
        rk[2 * r + 1] = k1;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
}
__device__ __forceinline__ uint4 philox_rk(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3, const uint32_t* rk) {
#pragma unroll
    for (int r = 0; r < 10; ++r) {
        uint32_t hi0 = __umulhi(0xD2511F53u, c0), lo0 = 0xD2511F53u * c0;
        uint32_t hi1 = __umulhi(0xCD9E8D57u, c2), lo1 = 0xCD9E8D57u * c2;
        uint32_t n0 = hi1 ^ c1 ^ rk[2 * r], n2 = hi0 ^ c3 ^ rk[2 * r + 1];
        c0 = n0; c1 = lo1; c2 = n2; c3 = lo0;
    }
    return make_uint4(c0, c1, c2, c3);
}

__device__ __forceinline__ uint32_t mulshift(uint32_t u, uint32_t n) {
    return (uint32_t)(((uint64_t)u * (uint64_t)n) >> 32);
}

// ---- Float functions of the sampling noise ---------------------------------
// Written so that the CPU oracle reproduces them bit for bit: every step is
// one IEEE round-to-nearest operation, spelled as an explicit intrinsic so
// the compiler fuses or reorders nothing, and the oracle performs the same
// steps in the same order.  Methods: the natural log by reduction to
// m in [sqrt(1/2), sqrt(2)), a 23-entry table of 32nds and the series of
// ln(1 + r) to r^5; cos(2 pi u) by quadrant and reflection to theta = (pi/2) h,
// h in [0, 1/2], and the Taylor series of cos (to theta^10) and sin (to
// theta^9); exp by z = k ln2 + r (k = rint(z log2 e), ln2 split in two) and
// the Taylor series of e^r to r^7, scaled by 2^k in the exponent field.
// Truncation errors are below 2e-9 (relative); rounding adds a few ulp.

// Uniform in the open interval: (w >> 9) + 1/2 over 2^23, a multiple of 2^-24
// in [2^-24, 1 - 2^-24] (exact in float, never 0 or 1).
__device__ __forceinline__ float unit_open(uint32_t w) {
    return __fmul_rn(__fadd_rn((float)(w >> 9), 0.5f), 0x1.0p-23f);
}

// ln x for a positive normal float x: x = 2^e m with m in [sqrt(1/2),
// sqrt(2)); c = 1 + i/32 is the nearest 32nd to m (i = rint(32 (m - 1)) in
// -9..13) and the table holds 1/c rounded to float (inv) and -ln(inv)
// rounded to float (L); then r = m inv - 1 (one rounding, |r| < 0.023) and
// ln x = e ln2 + L + ln(1 + r), the last by its Taylor series to r^5.  At
// i = 0 the table entry is exact (inv = 1, L = 0), so values near 1 keep
// their relative accuracy.
__device__ const float2 g_lntab[23] = {
    {0x1.642c86p+0f, -0x1.522ae2p-2f},
    {0x1.555556p+0f, -0x1.269624p-2f},
    {0x1.47ae14p+0f, -0x1.f991c4p-3f},
    {0x1.3b13b2p+0f, -0x1.a93ed8p-3f},
    {0x1.2f684cp+0f, -0x1.5bf408p-3f},
    {0x1.24924ap+0f, -0x1.1178eep-3f},
    {0x1.1a7b96p+0f, -0x1.9335e4p-4f},
    {0x1.111112p+0f, -0x1.08599ap-4f},
    {0x1.08421p+0f, -0x1.0415c8p-5f},
    {0x1p+0f, 0.0f},
    {0x1.f07c2p-1f, 0x1.f8299p-6f},
    {0x1.e1e1e2p-1f, 0x1.f0a30ap-5f},
    {0x1.d41d42p-1f, 0x1.6f0d28p-4f},
    {0x1.c71c72p-1f, 0x1.e27074p-4f},
    {0x1.bacf92p-1f, 0x1.29552cp-3f},
    {0x1.af286cp-1f, 0x1.5ff306p-3f},
    {0x1.a41a42p-1f, 0x1.9525a8p-3f},
    {0x1.99999ap-1f, 0x1.c8ff7ap-3f},
    {0x1.8f9c18p-1f, 0x1.fb918cp-3f},
    {0x1.861862p-1f, 0x1.1675cap-2f},
    {0x1.7d05f4p-1f, 0x1.2e8e2cp-2f},
    {0x1.745d18p-1f, 0x1.4618bap-2f},
    {0x1.6c16c2p-1f, 0x1.5d1bdap-2f},
};
__device__ __forceinline__ float xln(float x) {
    const uint32_t bx = __float_as_uint(x);
    const int e = (int)(bx - 0x3F3504F3u) >> 23;  // x / 2^e in [sqrt(1/2), sqrt(2))
    const float m = __uint_as_float(bx - ((uint32_t)e << 23));
    const int i = __float2int_rn(__fmul_rn(__fsub_rn(m, 1.0f), 32.0f));  // m - 1 and the scaling are exact
    const float2 t = __ldg(&g_lntab[i + 9]);
    const float r = __fmaf_rn(m, t.x, -1.0f);
    float p = 0x1.99999ap-3f;          // 1/5
    p = __fmaf_rn(p, r, -0.25f);
    p = __fmaf_rn(p, r, 0x1.555556p-2f);  // 1/3
    p = __fmaf_rn(p, r, -0.5f);
    p = __fmaf_rn(p, r, 1.0f);
    return __fmaf_rn((float)e, 0x1.62e43p-1f, __fmaf_rn(r, p, t.y));
}

// cos(2 pi u) for u in (0, 1) a multiple of 2^-24.
__device__ __forceinline__ float xcos2pi(float u) {
    const float v = __fmul_rn(u, 4.0f);  // exact
    const int q = (int)v;                // quadrant 0..3
    const float r = __fsub_rn(v, (float)q);
    const bool low = r <= 0.5f;
    const float h = low ? r : __fsub_rn(1.0f, r);
    const float y = __fmul_rn(h, h);
    float c = -0x1.a6d1f2p-16f;          // cos(pi h / 2) = sum (-1)^k (pi/2)^2k h^2k / (2k)!
    c = __fmaf_rn(c, y, 0x1.e1f506p-11f);
    c = __fmaf_rn(c, y, -0x1.55d3c8p-6f);
    c = __fmaf_rn(c, y, 0x1.03c1f0p-2f);
    c = __fmaf_rn(c, y, -0x1.3bd3ccp+0f);
    c = __fmaf_rn(c, y, 1.0f);
    float sn = 0x1.507834p-13f;          // sin(pi h / 2) = h sum (-1)^k (pi/2)^(2k+1) h^2k / (2k+1)!
    sn = __fmaf_rn(sn, y, -0x1.32d2ccp-8f);
    sn = __fmaf_rn(sn, y, 0x1.466bc6p-4f);
    sn = __fmaf_rn(sn, y, -0x1.4abbcep-1f);
    sn = __fmaf_rn(sn, y, 0x1.921fb6p+0f);
    sn = __fmul_rn(sn, h);
    const float cr = low ? c : sn, sr = low ? sn : c;  // cos / sin of (pi/2) r
    return q == 0 ? cr : (q == 1 ? -sr : (q == 2 ? -cr : sr));
}

// e^z for z <= 88 (0 below -80).
__device__ __forceinline__ float xexp(float z) {
    if (z < -80.0f) return 0.0f;
    const float k = rintf(__fmul_rn(z, 0x1.715476p+0f));
    float r = __fmaf_rn(-k, 0x1.62e43p-1f, z);
    r = __fmaf_rn(-k, -0x1.05c61p-29f, r);
    float p = 0x1.a01a02p-13f;  // 1/7!
    p = __fmaf_rn(p, r, 0x1.6c16c2p-10f);
    p = __fmaf_rn(p, r, 0x1.111112p-7f);
    p = __fmaf_rn(p, r, 0x1.555556p-5f);
    p = __fmaf_rn(p, r, 0x1.555556p-3f);
    p = __fmaf_rn(p, r, 0.5f);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    return __uint_as_float(__float_as_uint(p) + ((uint32_t)(int)k << 23));
}

__device__ __forceinline__ uint64_t warp_xor64(uint64_t v) {
    uint32_t lo = (uint32_t)v, hi = (uint32_t)(v >> 32);
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        lo ^= __shfl_xor_sync(FULL, lo, o);
        hi ^= __shfl_xor_sync(FULL, hi, o);
    }
    return ((uint64_t)hi << 32) | lo;
}

__device__ __forceinline__ int warp_sum(int v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(FULL, v, o);
    return v;
}

// ---- bulk async copies shared -> global (TMA engine, no multicast) --------
__device__ __forceinline__ void bulk_s2g(void* gdst, const void* ssrc, uint32_t bytes) {
    uint32_t s = (uint32_t)__cvta_generic_to_shared(ssrc);
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gdst), "r"(s), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// Orders async-proxy (bulk copy) and generic-proxy accesses to global memory.
__device__ __forceinline__ void fence_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }
// Makes generic-proxy writes to shared memory visible to later bulk copies.
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ---- mbarriers (CTA shared memory) and global -> shared bulk loads --------
__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
// Makes mbarrier initialisation visible to the async proxy (bulk copies).
__device__ __forceinline__ void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.release.cta.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
                 : "memory");
}
// One arrival that also expects `bytes` of bulk-copy transactions.
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.release.cta.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                     smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return done != 0;
}
// Waits for the phase of parity `parity` to complete, for at most about
// `limit_ns` of wall time; false if it gave up.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint64_t limit_ns = 1000000000ull) {
    if (mbar_test(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    while (!mbar_test(bar, parity))
        if (global_ns() - t0 > limit_ns) return false;
    return true;
}
// Bulk copy global -> this CTA's shared memory, completing on `bar`
// (16-byte aligned addresses, size a multiple of 16; no multicast).
__device__ __forceinline__ void bulk_g2s(void* sdst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(sdst)),
                 "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

// Three bits of a Zobrist hash in a 64-bit Bloom filter (the hash bits are
// uniformly random, so its low 18 bits serve as three independent indices).
__device__ __forceinline__ uint64_t bloom_bits(uint64_t h) {
    return (1ull << (h & 63)) | (1ull << ((h >> 6) & 63)) | (1ull << ((h >> 12) & 63));
}

}  // namespace sb
