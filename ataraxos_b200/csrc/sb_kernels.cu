// sb_kernels.cu -- B200 kernels and C ABI of the Stratego rollout simulator.
//
// The hot path is env_kernel<T, MODE>: one warp per env, one launch per ply
// (or k plies per launch for the trajectory ring), doing action sampling,
// move validation / combat / trackers / terminal check, auto-reset from the
// setup pool, and the observation outputs of the new state (legal mask,
// 488-channel infostate) in a single pass over the env's 256-byte record
// staged in shared memory.  Output rows are stored straight from registers
// as whole rows; in the single-ply production step a producer warp per CTA
// streams the move-history planes' zero rows with bulk asynchronous copies
// (cp.async.bulk.global.shared::cta, the TMA engine, no multicast) while the
// other warps play, and the history's +1 / -1 land on top after an mbarrier
// handshake.
//
// Semantics follow the reference simulator csrc/stratego_buffer.cu (cited per
// function) with the Zobrist hash kept incrementally in the record instead of
// being recomputed over 100 squares.
#include <stdarg.h>
#include <stdio.h>
#include <string.h>
#include <time.h>

#include <atomic>
#include <mutex>

#include "sb_device.cuh"
#include "stratego_b200.h"

namespace sb {

enum : uint32_t {
    F_RESET_PLANES = 1u << 0,  // reset from setup planes (reference reset_terminated)
    F_RESET_POOL = 1u << 1,    // reset from the setup pool
    F_FORCE = 1u << 2,         // reset every env, not only terminated ones
    F_APPLY = 1u << 3,         // apply one action per env
    F_STEP = 1u << 4,          // step() semantics: stuck rule, transition outputs
    F_AUTO_RESET = 1u << 5,    // after apply, reset terminated envs from the pool
    F_PROPOSE = 1u << 6,       // cache a proposal for the new state at propose_ply
    F_MASK_U8 = 1u << 7,
    F_MASK_BITS = 1u << 8,
    F_INFO = 1u << 9,
    F_HAS_LEGAL = 1u << 10,
    F_HASH = 1u << 11,
    F_SAMPLE_OUT = 1u << 12,   // write the sampled action of the current state
};

struct KArgs {
    uint8_t* rec;
    int64_t* ring;
    const int64_t* zob;
    const uint8_t* pool;
    int64_t pool_size;
    int64_t n;
    int64_t env_base;
    uint64_t seed;
    uint32_t rk[20];  // Philox round keys of `seed` (philox_round_keys)
    int32_t no_attack_limit, max_len, ts_limit, policy;
    int32_t* status;
    const float* logits;
    uint32_t flags;
    int32_t info_layout;
    const int64_t* actions;
    int64_t ply;
    int64_t propose_ply;
    const int8_t* setup_red;
    const int8_t* setup_blue;
    uint8_t* mask_u8;
    uint8_t* mask_bits;
    void* info;
    float* reward;
    uint8_t* done;
    int64_t* action_taken;
    float* logprob_taken;
    int16_t* next_action;
    float* next_logprob;
    int64_t* hash;
    uint8_t* has_legal;
    int64_t* stats;
    int64_t* sampled;
    float* sampled_lp;
    int32_t sm_warp;
    // step modes: plies per launch (0 = observe only) and the output ring.
    // Ply p of a launch reads its transition outputs (reward, done, taken
    // action) at slot (slot0 + p) % n_slots and writes the observation of the
    // new state (mask, infostate, proposal, hash) at slot (slot0 + p + 1) %
    // n_slots; every output array is laid out [n_slots, n, ...].  The host
    // passes slot0 already reduced (0 <= slot0 < n_slots < 2^31), so the
    // kernel walks the ring with counters instead of dividing.
    int32_t n_plies;
    int32_t n_slots;
    int32_t slot0;
    int32_t rules;  // SB_RULES_*
    uint8_t* isf;   // [n, ISF_TS_BYTES] under SB_RULES_ISF
    // step server (MODE_SERVE): control block in mapped page-locked host
    // memory (SERVE_GO, SERVE_STOP, SERVE_DONE), its device relay
    // (SERVE_GO, SERVE_STOP, DEV_DONE_COUNT), the device result block copied
    // to page-locked host memory after every step, and the longest a CTA
    // waits for the host's next step
    int64_t* serve_ctl;
    int64_t* serve_dev;
    const uint8_t* serve_back_dev;
    uint8_t* serve_back_host;
    int64_t serve_back_bytes;
    int64_t serve_limit_ns;
};

constexpr int SERVE_GO = 0, SERVE_STOP = 1, SERVE_DONE = 16, DEV_DONE_COUNT = 2;

constexpr int WARPS = 8;  // warps (envs in flight) per CTA
constexpr int ZOB_N = 2600;  // entries of the [10,10,2,13] Zobrist table
constexpr int SM_RAYS = 256;   // 100 x uint16 packed rays
constexpr int SM_SCRATCH = 576;  // 512-byte scratch: the Gumbel sampler's per-square move-count prefix
constexpr int SM_FIXED = 1088;
constexpr int SM_BITS = SM_FIXED;  // 1264-byte bit-packed legal mask (mask outputs only)
constexpr int ZERO_BYTES = 12800;  // MODE_STEP_PROD: per-CTA zero buffer, source of the bulk zero rows

// ---------------------------------------------------------------------------
// Legal moves
// ---------------------------------------------------------------------------

// Move generation on bitboards.  The 100 squares form two 128-bit boards
// held in four registers each, row-major (square r*10+c) and column-major
// (index c*10+r), built with ballots.  A piece's four rays are ffs / clz
// searches on the 10-bit line of its row or column: stoppers S (own pieces
// and lakes: neither entered nor passed) and enemies E (entered, end the
// slide); non-scouts keep one square (csrc/stratego_buffer.cu:467-506).

// Lakes: squares 42,43,46,47,52,53,56,57 (stratego/constants.py:25-28), and
// their column-major indices 24,25,34,35,64,65,74,75.
__device__ __forceinline__ uint32_t lake_word(int k) { return k == 1 ? 0x0330CC00u : 0u; }
__device__ __forceinline__ uint32_t lake_word_t(int k) { return k == 0 ? 0x03000000u : (k == 1 ? 0x0000000Cu : (k == 2 ? 0x00000C03u : 0u)); }

// The 10 bits of a 128-bit board (w0..w3) that start at bit pos (a multiple of 10).
__device__ __forceinline__ uint32_t line10(uint32_t w0, uint32_t w1, uint32_t w2, uint32_t w3, int pos) {
    const int i = pos >> 5;
    const uint32_t lo = i == 0 ? w0 : (i == 1 ? w1 : (i == 2 ? w2 : w3));
    const uint32_t hi = i == 0 ? w1 : (i == 1 ? w2 : (i == 2 ? w3 : 0u));
    return __funnelshift_r(lo, hi, pos & 31) & 0x3FFu;
}
// Squares reachable from position x of a line towards higher positions ...
__device__ __forceinline__ int ray_fwd(uint32_t S, uint32_t E, int x) {
    const uint32_t m = ((S | E) >> (x + 1)) & ((1u << (9 - x)) - 1u);
    if (!m) return 9 - x;
    const int f = __ffs(m) - 1;
    return f + (int)((E >> (x + 1 + f)) & 1u);
}
// ... and towards lower positions.
__device__ __forceinline__ int ray_back(uint32_t S, uint32_t E, int x) {
    const uint32_t m = (S | E) & ((1u << x) - 1u);
    if (!m) return x;
    const int h = 31 - __clz(m);
    return (x - 1 - h) + (int)((E >> h) & 1u);
}

// Position of the k-th (0-based) set bit of m (popcount bisection).
__device__ __forceinline__ int nth_bit(uint32_t m, int k) {
    int pos = 0, c = __popc(m & 0xFFFFu);
    if (k >= c) { k -= c; m >>= 16; pos += 16; }
    c = __popc(m & 0xFFu);
    if (k >= c) { k -= c; m >>= 8; pos += 8; }
    c = __popc(m & 0xFu);
    if (k >= c) { k -= c; m >>= 4; pos += 4; }
    c = __popc(m & 0x3u);
    if (k >= c) { k -= c; m >>= 2; pos += 2; }
    return pos + (k >= (int)(m & 1u) ? 1 : 0);
}

// Ray lengths of every square for side p, packed as up | left<<4 | right<<8
// | down<<12 (the groups in ascending destination order) into rays[] (0 for
// squares without a movable piece of side p); returns the number of legal
// moves (warp-uniform).  The rays are computed per movable piece: lane i
// takes the i-th movable piece in ascending square order (a second round
// when there are more than 32), so the ray arithmetic runs once or twice
// per warp instead of once per 32-square block.
// Not inlined: its call sites share one copy of the code, which keeps the
// step kernel's instruction footprint small.
__device__ __noinline__ int enumerate(const uint8_t* b, int p, uint16_t* rays, int lane) {
    uint32_t own[4], opp[4], ownT[4], oppT[4], mv[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int i = lane + 32 * k;
        const uint8_t c = i < NSQ ? b[i] : 0;
        const uint8_t ct = i < NSQ ? b[(i % 10) * 10 + i / 10] : 0;
        const bool co = c & C_OCC, cto = ct & C_OCC;
        const bool cm = co && ((c >> 4) & 1) == p, ctm = cto && ((ct >> 4) & 1) == p;
        own[k] = __ballot_sync(FULL, cm);
        opp[k] = __ballot_sync(FULL, co && !cm);
        ownT[k] = __ballot_sync(FULL, ctm);
        oppT[k] = __ballot_sync(FULL, cto && !ctm);
        mv[k] = __ballot_sync(FULL, cm && can_move(c & C_PIECE));
    }
    // lane l (l = lane % 10) extracts row l and column l as 10-bit lines,
    // stoppers | enemies << 16; a piece fetches its row and column line with
    // one shuffle each
    const int l = lane % 10;
    const uint32_t rw = line10(own[0] | lake_word(0), own[1] | lake_word(1), own[2] | lake_word(2),
                               own[3] | lake_word(3), 10 * l) |
                        (line10(opp[0], opp[1], opp[2], opp[3], 10 * l) << 16);
    const uint32_t cw = line10(ownT[0] | lake_word_t(0), ownT[1] | lake_word_t(1), ownT[2] | lake_word_t(2),
                               ownT[3] | lake_word_t(3), 10 * l) |
                        (line10(oppT[0], oppT[1], oppT[2], oppT[3], 10 * l) << 16);
    for (int i = lane; i < NSQ / 2; i += 32) reinterpret_cast<uint32_t*>(rays)[i] = 0u;
    __syncwarp();
    const int c0 = __popc(mv[0]), c01 = c0 + __popc(mv[1]), c012 = c01 + __popc(mv[2]);
    const int npieces = c012 + __popc(mv[3]);
    int total = 0;
    for (int base = 0; base < npieces; base += 32) {
        const int i = base + lane;
        int sq = -1;
        if (i < npieces) {
            const int w = i < c0 ? 0 : (i < c01 ? 1 : (i < c012 ? 2 : 3));
            const int k = i - (w == 0 ? 0 : (w == 1 ? c0 : (w == 2 ? c01 : c012)));
            const uint32_t m = w == 0 ? mv[0] : (w == 1 ? mv[1] : (w == 2 ? mv[2] : mv[3]));
            sq = 32 * w + nth_bit(m, k);
        }
        const int r = sq >= 0 ? sq / 10 : 0, col = sq >= 0 ? sq - 10 * r : 0;
        const uint32_t rl = __shfl_sync(FULL, rw, r), cl = __shfl_sync(FULL, cw, col);
        if (sq >= 0) {
            const uint32_t rs = rl & 0x3FFu, re = rl >> 16, cs = cl & 0x3FFu, ce = cl >> 16;
            int up = ray_back(cs, ce, r), down = ray_fwd(cs, ce, r);
            int left = ray_back(rs, re, col), right = ray_fwd(rs, re, col);
            if ((b[sq] & C_PIECE) != 2) {
                up = min(up, 1);
                down = min(down, 1);
                left = min(left, 1);
                right = min(right, 1);
            }
            rays[sq] = (uint16_t)(up | (left << 4) | (right << 8) | (down << 12));
            total += up + left + right + down;
        }
    }
    total = __reduce_add_sync(FULL, total);
    __syncwarp();
    return total;
}

// Moves of a packed ray set, and of the lane's four squares.
__device__ __forceinline__ int ray_count(uint32_t r) { return (r & 15) + ((r >> 4) & 15) + ((r >> 8) & 15) + (r >> 12); }
__device__ __forceinline__ void ray_counts(const uint16_t* rays, int lane, int cnt[4]) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int sq = lane + 32 * k;
        cnt[k] = sq < NSQ ? ray_count(rays[sq]) : 0;
    }
}

// j-th destination (0-based, ascending) of a packed ray set.
__device__ __forceinline__ int decode_ray(int sq, uint32_t r, int j) {
    const int up = r & 15, left = (r >> 4) & 15, right = (r >> 8) & 15;
    if (j < up) return sq - 10 * (up - j);
    j -= up;
    if (j < left) return sq - (left - j);
    j -= left;
    if (j < right) return sq + 1 + j;
    j -= right;
    return sq + 10 * (1 + j);
}

// kth legal action in ascending src*100+dst order (warp-uniform result).
// The four 32-square blocks are scanned together, two 16-bit sums per word.
__device__ int kth_action(int kth, const uint16_t* rays, int lane) {
    int cnt[4];
    ray_counts(rays, lane, cnt);
    uint32_t a01 = (uint32_t)cnt[0] | ((uint32_t)cnt[1] << 16), a23 = (uint32_t)cnt[2] | ((uint32_t)cnt[3] << 16);
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t v01 = __shfl_up_sync(FULL, a01, o), v23 = __shfl_up_sync(FULL, a23, o);
        if (lane >= o) {
            a01 += v01;
            a23 += v23;
        }
    }
    const uint32_t t01 = __shfl_sync(FULL, a01, 31), t23 = __shfl_sync(FULL, a23, 31);
    const int b1 = (int)(t01 & 0xFFFF), b2 = b1 + (int)(t01 >> 16), b3 = b2 + (int)(t23 & 0xFFFF);
    const int k = kth < b1 ? 0 : (kth < b2 ? 1 : (kth < b3 ? 2 : 3));
    const int base = k == 0 ? 0 : (k == 1 ? b1 : (k == 2 ? b2 : b3));
    const uint32_t aw = k < 2 ? a01 : a23;
    const int incl = (int)(k & 1 ? aw >> 16 : aw & 0xFFFF);
    const int c = k == 0 ? cnt[0] : (k == 1 ? cnt[1] : (k == 2 ? cnt[2] : cnt[3]));
    const unsigned m = __ballot_sync(FULL, kth < base + incl);
    if (!m) return -1;
    const int L = __ffs(m) - 1;
    const int excl = __shfl_sync(FULL, incl - c, L);
    const int sq = L + 32 * k;
    return sq * 100 + decode_ray(sq, rays[sq], kth - base - excl);
}


// Choose an action for the current state (rays already enumerated, n moves).
// Uniform: k = (u32 * n) >> 32 over ascending legal actions, log-prob -ln n.
// Softmax policy (SB_POLICY_GUMBEL): action a has logit z_a (from memory, or
// virtual N(0,1): Box-Muller on Philox(seed; env, ply, a, TAG_LOGIT) words
// x, y) and an Exp(1) variate E_a = -ln(word z); the choice is the legal a
// with the largest q_a / E_a, q_a = e^(z_a - c) (c = 0 for virtual logits,
// the legal maximum for logits in memory), ties to the smaller action index;
// a beats b when q_a E_b > q_b E_a (two rounded products, no division).
// That is Gumbel-max: ln(q_a / E_a) = z_a - c + G_a with G_a = -ln E_a
// Gumbel(0,1), so a is drawn from the softmax of the legal logits.  The
// log-prob is z_a - c - ln(sum of q over legal actions).  The order of the
// sum and of the comparisons is fixed: lane L takes the L-th, (L+32)-th, ...
// legal action (ascending order) in that order, then a butterfly over the
// lanes (xor 16, 8, 4, 2, 1); with the float functions above, every value is
// reproduced bit for bit by the CPU oracle.
// acts: the warp's shared-memory scratch (at least 200 bytes).
// u_pre: the uniform policy's Philox word when the caller drew it already.
struct Pick {
    const uint32_t* rk;   // Philox round keys (in the kernel's parameter block)
    int64_t env_base;
    const float* logits;  // [n,10000] or nullptr (virtual N(0,1) logits)
    int policy;
};

template <int POL>
__device__ void choose(const Pick& a, const uint16_t* rays, int n, int64_t e, int64_t ply,
                       int lane, int& act, float& lp, uint16_t* scratch = nullptr, const uint32_t* u_pre = nullptr) {
    const int64_t ge = a.env_base + e;
    if (n == 0) {
        act = -1;
        lp = 0.0f;
        return;
    }
    const int pol = POL >= 0 ? POL : a.policy;
    if (pol == SB_POLICY_UNIFORM) {
        const uint32_t u =
            u_pre ? *u_pre : philox_rk((uint32_t)ge, (uint32_t)ply, (uint32_t)((uint64_t)ply >> 32), TAG_ACTION, a.rk).x;
        act = kth_action((int)mulshift(u, (uint32_t)n), rays, lane);
        lp = -xln((float)n);
        return;
    }
    int cnt[4];
    ray_counts(rays, lane, cnt);
    // Lane L takes the L-th, (L+32)-th, ... legal action in ascending order:
    // the inclusive prefix of the per-square move counts goes to shared
    // memory, and each lane finds the square of its action by binary search
    // (the first square whose prefix exceeds the action's rank).
    uint16_t* incl16 = scratch;  // [100]
    {
        int base = 0;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int c = cnt[k];
            int incl = c;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int v = __shfl_up_sync(FULL, incl, o);
                if (lane >= o) incl += v;
            }
            const int sq = lane + 32 * k;
            if (sq < NSQ) incl16[sq] = (uint16_t)(base + incl);
            base += __shfl_sync(FULL, incl, 31);
        }
        __syncwarp();
    }
    const float* lg = a.logits ? a.logits + e * NACT : nullptr;
    float shift = 0.0f;  // c: 0, or the legal maximum of the logits in memory
    float bq = 0.0f, bE = 1.0f, bestz = 0.0f, s = 0.0f;  // the lane's best so far: q, E, logit
    int besta = 0x7fffffff;
    // pass 0 (logits in memory only): their legal maximum; pass 1: the choice
#pragma unroll 1
    for (int pass = lg ? 0 : 1; pass < 2; ++pass) {
        float mx = -INFINITY;
#pragma unroll 1
        for (int t = lane; t < n; t += 32) {
            int lo = 0, hi = NSQ - 1;
#pragma unroll
            for (int it = 0; it < 7; ++it) {  // 2^7 >= 100 squares
                const int mid = (lo + hi) >> 1;
                if ((int)incl16[mid] > t) hi = mid;
                else lo = mid + 1;
            }
            const uint32_t r = rays[lo];
            const int ac = lo * 100 + decode_ray(lo, r, t - ((int)incl16[lo] - ray_count(r)));
            if (pass == 0) {
                mx = fmaxf(mx, lg[ac]);
                continue;
            }
            const uint4 w = philox_rk((uint32_t)ge, (uint32_t)ply, (uint32_t)ac, TAG_LOGIT, a.rk);
            const float z = lg ? lg[ac]
                               : __fmul_rn(__fsqrt_rn(__fmul_rn(-2.0f, xln(unit_open(w.x)))), xcos2pi(unit_open(w.y)));
            const float q = xexp(__fsub_rn(z, shift));
            const float E = -xln(unit_open(w.z));
            const float lhs = __fmul_rn(q, bE), rhs = __fmul_rn(bq, E);
            if (lhs > rhs || (lhs == rhs && ac < besta)) {
                bq = q;
                bE = E;
                besta = ac;
                bestz = z;
            }
            s = __fadd_rn(s, q);
        }
        if (pass == 0) {
#pragma unroll
            for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(FULL, mx, o));
            shift = mx;
        }
    }
    __syncwarp();
#pragma unroll 1
    for (int o = 16; o; o >>= 1) {
        const float oq = __shfl_xor_sync(FULL, bq, o), oE = __shfl_xor_sync(FULL, bE, o);
        const float oz = __shfl_xor_sync(FULL, bestz, o);
        const int oa = __shfl_xor_sync(FULL, besta, o);
        const float lhs = __fmul_rn(oq, bE), rhs = __fmul_rn(bq, oE);
        if (lhs > rhs || (lhs == rhs && oa < besta)) {
            bq = oq;
            bE = oE;
            besta = oa;
            bestz = oz;
        }
        s = __fadd_rn(s, __shfl_xor_sync(FULL, s, o));
    }
    act = besta;
    lp = __fsub_rn(__fsub_rn(bestz, shift), xln(s));
}

// choose() for the start of a ply whose proposal was not cached (after a
// host-side change of the state, or logits in memory): one out-of-line copy,
// so the hot per-ply proposal keeps the kernel's instruction footprint.
// The policy's inputs come as scalars (not the kernel's argument block,
// whose address would need a local-memory copy).
template <int POL>
__device__ __noinline__ void choose_cold(const uint32_t* rk, int64_t env_base, const float* logits, int policy,
                                         const uint16_t* rays, int n, int64_t e, int64_t ply, int lane, int& act,
                                         float& lp, uint16_t* scratch) {
    choose<POL>(Pick{rk, env_base, logits, policy}, rays, n, e, ply, lane, act, lp, scratch);
}

// ---------------------------------------------------------------------------
// Reset (csrc/stratego_buffer.cu:529-618; host part cpp:289-291)
// ---------------------------------------------------------------------------

// zt: the Zobrist table (the CTA's shared-memory copy in env_kernel).
// isf: the ISF repetition rules are on (a.rules == SB_RULES_ISF; a constant
// false in the kernel modes that never run them).
__device__ void reset_env(uint8_t* rec, int64_t* ring2, const KArgs& a, const int64_t* zt, int64_t e, bool from_pool,
                          int lane, bool isf) {
    const uint8_t* red = nullptr;
    const uint8_t* blue = nullptr;
    const int32_t ep = fld<int32_t>(rec, R_EPISODE);
    if (from_pool) {
        const int64_t ge = a.env_base + e;
        const uint4 w = philox_rk((uint32_t)ge, (uint32_t)ep, (uint32_t)((uint64_t)ge >> 32), TAG_RESET, a.rk);
        const uint64_t ri = ((uint64_t)w.x * (uint64_t)a.pool_size) >> 32;
        const uint64_t bi = ((uint64_t)w.y * (uint64_t)a.pool_size) >> 32;
        red = a.pool + ri * 40;
        blue = a.pool + bi * 40;
    }
    uint64_t h = 0;
    bool bad = false;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int sq = lane + 32 * k;
        if (sq >= NSQ) continue;
        int rp, bp;
        if (from_pool) {
            rp = sq < 40 ? red[sq] : 0;
            bp = sq >= 60 ? blue[sq - 60] : 0;
        } else {
            rp = a.setup_red[e * NSQ + sq];
            bp = a.setup_blue[e * NSQ + sq];
        }
        uint8_t code = 0;
        if (rp != 0) {
            if (rp < 0 || rp > 12) bad = true;
            else {
                code = (uint8_t)(rp | C_OCC);
                h ^= zob(zt, sq, 0, rp);
            }
        } else if (bp != 0) {
            if (bp < 0 || bp > 12) bad = true;
            else {
                code = (uint8_t)(bp | C_OCC | C_BLUE);
                h ^= zob(zt, sq, 1, bp);
            }
        }
        rec[sq] = code;
    }
    h = warp_xor64(h);
    if (__any_sync(FULL, bad) && lane == 0 && a.status) atomicOr(a.status, SB_STATUS_BAD_SETUP);
    int4* rg = reinterpret_cast<int4*>(ring2);  // 2 x 64 x 8 B = 64 x 16 B
    rg[lane] = make_int4(0, 0, 0, 0);
    rg[lane + 32] = make_int4(0, 0, 0, 0);
    if (lane < 4) reinterpret_cast<int4*>(rec + R_HIST)[lane] = make_int4(0, 0, 0, 0);
    if (isf) {
        uint2* t = reinterpret_cast<uint2*>(a.isf + e * ISF_TS_BYTES);
        for (int i = lane; i < ISF_TS_BYTES / 8; i += 32) t[i] = make_uint2(~0u, ~0u);
    }
    if (lane == 0) {
        fld<int8_t>(rec, R_PLAYER) = 0;
        fld<int8_t>(rec, R_OUTCOME) = -1;
        rec[R_TERM] = 0;
        rec[R_FLAGCAP] = 0;
        fld<int32_t>(rec, R_MOVENUM) = 0;
        fld<int32_t>(rec, R_MSA) = 0;
        fld<int32_t>(rec, R_TSINCE) = 0;
        rec[R_HHEAD] = 0;
        rec[R_HLEN] = 0;
        rec[R_TSVIOL] = 0;
        rec[R_CHVIOL] = 0;
        if (isf) {
            fld<uint64_t>(rec, R_ISF_THR) = ~0ull;
            fld<uint64_t>(rec, R_ISF_EV) = ~0ull << 8;  // evasion bits clear, spare bytes 0xFF
        } else {
            fld<int32_t>(rec, R_TSCOUNT) = 0;
            fld<int32_t>(rec, R_TSCOUNT + 4) = 0;
            fld<int16_t>(rec, R_TSLO) = -1;
            fld<int16_t>(rec, R_TSLO + 2) = -1;
            fld<int16_t>(rec, R_TSHI) = -1;
            fld<int16_t>(rec, R_TSHI + 2) = -1;
        }
        rec[R_CHHEAD] = 0;
        rec[R_CHHEAD + 1] = 0;
        rec[R_CHLEN] = 0;
        rec[R_CHLEN + 1] = 0;
        fld<int8_t>(rec, R_CHLAST) = -1;
        fld<int8_t>(rec, R_CHLAST + 1) = -1;
        fld<int16_t>(rec, R_PROP) = -1;
        fld<uint64_t>(rec, R_ZHASH) = h;
        fld<int32_t>(rec, R_EPISODE) = ep + (from_pool ? 1 : 0);
        fld<int32_t>(rec, R_PROPPLY) = -1;
        fld<int16_t>(rec, R_NLEGAL) = 0;
        fld<float>(rec, R_PROPLP) = 0.0f;
        fld<uint64_t>(rec, R_BLOOM) = 0;
        fld<uint64_t>(rec, R_BLOOM + 8) = 0;
    }
    __syncwarp();
}

// ---------------------------------------------------------------------------
// Apply one action (csrc/stratego_buffer.cu:111-399)
// ---------------------------------------------------------------------------

// ISF two-square state: per square the (lo, hi) intervals of one row or
// column that the piece there covered in its last 1, 2, 3 moves in a row (the
// intersections of its last k segments), as u16 lo | hi << 8, 0xFFFF when
// fewer than two squares remain (stratego/env/two_square.py:27-94: the pairs
// counted k times are exactly the pairs inside that interval).
__device__ __forceinline__ uint32_t iv_and(uint32_t x, uint32_t y) {
    if (x == 0xFFFFu || y == 0xFFFFu) return 0xFFFFu;
    const int xl = x & 0xFF, xh = x >> 8, yl = y & 0xFF, yh = y >> 8;
    const int xline = xl / 10 == xh / 10 ? xl / 10 : 10 + xl % 10;
    const int yline = yl / 10 == yh / 10 ? yl / 10 : 10 + yl % 10;
    if (xline != yline) return 0xFFFFu;
    const int lo = max(xl, yl), hi = min(xh, yh);
    return lo < hi ? (uint32_t)(lo | (hi << 8)) : 0xFFFFu;
}

// Returns false (and changes nothing) when the action is rejected.  On
// success the board, counters, history, trackers and the caps part of the
// terminal check are done; check_legal asks the caller for the "side to move
// has no legal move" test on the new board.
// The chase ring is read only when the mover's Bloom filter of its hashes
// (R_BLOOM, cleared with the ring) says the new hash may be in it.
// tsq: the env's ISF two-square state, or nullptr when the ISF rules are off.
__device__ bool apply_env(uint8_t* rec, int64_t* ring2, const KArgs& a, const int64_t* zt, int64_t act, int lane,
                          bool& check_legal, bool& flag_taken, uint8_t* tsq) {
    check_legal = false;
    flag_taken = false;
    if (act < 0 || act >= NACT) return false;
    const int p = fld<int8_t>(rec, R_PLAYER);
    const int src = (int)act / 100, dst = (int)act % 100;
    if (src == dst) return false;
    const uint8_t cs = rec[src], cd = rec[dst];
    const int ps = cs & C_PIECE, pd = cd & C_PIECE;
    if (!(cs & C_OCC) || ((cs >> 4) & 1) != p || !can_move(ps)) return false;
    if ((cd & C_OCC) && ((cd >> 4) & 1) == p) return false;
    if (is_lake(dst)) return false;
    const int sr = src / 10, sc = src % 10, dr = dst / 10, dc = dst % 10;
    if (sr != dr && sc != dc) return false;
    if (ps != 2) {
        const int dist = sr != dr ? abs(dr - sr) : abs(dc - sc);
        if (dist != 1) return false;
    } else {
        const int step = sr != dr ? (dr > sr ? 10 : -10) : (dc > sc ? 1 : -1);
        for (int q = src + step; q != dst; q += step)
            if (is_lake(q) || (rec[q] & C_OCC)) return false;
    }
    const int opp = 1 - p;
    const bool attack = (cd & C_OCC) != 0;
    // 0 plain move, 1 attacker wins, 2 defender wins, 3 both removed
    int result;
    int8_t outcome = fld<int8_t>(rec, R_OUTCOME);
    if (!attack) result = 0;
    else if (pd == 11) {
        result = 1;
        flag_taken = true;
        outcome = (int8_t)(p == 0 ? 0 : 1);
    } else if (pd == 12) result = ps == 3 ? 1 : 2;
    else if (ps == 1 && pd == 10) result = 1;
    else result = ps > pd ? 1 : (ps < pd ? 2 : 3);

    // moved / revealed flags (cu:243-253)
    uint8_t fs, fd;
    if (attack) {
        fs = (uint8_t)((cs & C_MOVED) | C_REV);
        fd = (uint8_t)((cd & C_MOVED) | C_REV);
    } else {
        fs = C_MOVED;
        fd = (uint8_t)(C_MOVED | (cs & C_REV));
    }
    uint8_t dpart = 0;
    if (result <= 1) dpart = (uint8_t)(ps | C_OCC | (p ? C_BLUE : 0));
    else if (result == 2) dpart = (uint8_t)(cd & (C_PIECE | C_BLUE | C_OCC));
    const uint8_t ns = fs, nd = (uint8_t)(fd | dpart);

    uint64_t h = fld<uint64_t>(rec, R_ZHASH) ^ zob(zt, src, p, ps);
    if (result == 0) h ^= zob(zt, dst, p, ps);
    else if (result == 1) h ^= zob(zt, dst, opp, pd) ^ zob(zt, dst, p, ps);
    else if (result == 3) h ^= zob(zt, dst, opp, pd);

    const int32_t msa = attack ? 0 : fld<int32_t>(rec, R_MSA) + 1;
    const int32_t mn = fld<int32_t>(rec, R_MOVENUM) + 1;
    const int head = rec[R_HHEAD], hlen = rec[R_HLEN];

    const bool isf = tsq != nullptr;
    const uint64_t h_before = fld<uint64_t>(rec, R_ZHASH);
    uint8_t tsv = rec[R_TSVIOL];
    uint8_t chv = rec[R_CHVIOL];

    // two-square
    int32_t tsc = 0;
    int tslo = -1, tshi = -1;
    uint32_t isf_new[3] = {0xFFFFu, 0xFFFFu, 0xFFFFu};  // ISF: the entry the piece carries to dst
    bool isf_keep_dst = false;
    if (!isf) {
        // per mover (cu:272-296)
        tsc = fld<int32_t>(rec, R_TSCOUNT + 4 * p);
        tslo = fld<int16_t>(rec, R_TSLO + 2 * p);
        tshi = fld<int16_t>(rec, R_TSHI + 2 * p);
        if (attack) {
            tsc = 0;
            tslo = -1;
            tshi = -1;
        } else {
            const int lo = min(src, dst), hi = max(src, dst);
            if (tslo == lo && tshi == hi) ++tsc;
            else {
                tsc = 1;
                tslo = lo;
                tshi = hi;
            }
            if (tsc > a.ts_limit) tsv = 1;
        }
    } else if (!attack) {
        // per piece (two_square.py:27-63): the move breaks the rule when the
        // piece's last `limit` segments still share two squares with it
        const uint16_t* t = reinterpret_cast<const uint16_t*>(tsq) + src * 3;
        const uint32_t i1 = t[0], i2 = t[1], i3 = t[2];
        const uint32_t seg = (uint32_t)min(src, dst) | ((uint32_t)max(src, dst) << 8);
        const uint32_t il = a.ts_limit == 1 ? i1 : (a.ts_limit == 2 ? i2 : i3);
        if (iv_and(il, seg) != 0xFFFFu) tsv = 1;
        isf_new[0] = seg;
        isf_new[1] = iv_and(seg, i1);
        isf_new[2] = iv_and(seg, i2);
    } else {
        // an attack is exempt: the attacker arrives with no counters, a
        // surviving defender keeps its own
        isf_keep_dst = result == 2;
    }

    // chasing: the opponent pieces 4-adjacent to dst on the new board
    // (cu:306-381; chasing.py:115-125), in the order up, down, left, right
    bool threat = false;
    uint32_t thr = ~0u;
    int nt = 0;
#pragma unroll
    for (int d = 0; d < 4; ++d) {
        int q;
        if (d == 0) { if (dr == 0) continue; q = dst - 10; }
        else if (d == 1) { if (dr == 9) continue; q = dst + 10; }
        else if (d == 2) { if (dc == 0) continue; q = dst - 1; }
        else { if (dc == 9) continue; q = dst + 1; }
        if (is_lake(q)) continue;
        const uint8_t c = q == src ? ns : rec[q];
        if ((c & C_OCC) && ((c >> 4) & 1) == opp) {
            threat = true;
            thr = (thr & ~(0xFFu << (8 * nt))) | ((uint32_t)q << (8 * nt));
            ++nt;
        }
    }
    int chh = rec[R_CHHEAD + p], chl = rec[R_CHLEN + p], chlast = fld<int8_t>(rec, R_CHLAST + p);
    uint64_t bloom = fld<uint64_t>(rec, R_BLOOM + 8 * p);
    int64_t* ring = ring2 + p * NRING;
    auto ring_has = [&](uint64_t x) -> bool {
        const uint64_t bb = bloom_bits(x);
        if ((bloom & bb) != bb) return false;
        const bool f = (lane < chl && (uint64_t)ring[lane] == x) || (lane + 32 < chl && (uint64_t)ring[lane + 32] == x);
        return __any_sync(FULL, f);
    };
    auto ring_add = [&](uint64_t x) {
        bloom |= bloom_bits(x);
        if (lane == 0) ring[chl < NRING ? chl : chh] = (int64_t)x;
        if (chl < NRING) ++chl;
        else chh = (chh + 1) % NRING;
    };
    uint8_t evb = 0;
    if (!isf) {
        // every threatening move is part of the chase; a repeated position
        // breaks the rule unless dst is the square last left
        if (threat) {
            const bool found = ring_has(h);
            const bool exc = chlast >= 0 && dst == chlast;
            if (found && !exc) chv = 1;
            ring_add(h);
            chlast = src;
        } else {
            chl = 0;
            chh = 0;
            chlast = -1;
            bloom = 0;
        }
    } else {
        // evasion-gated (chasing.py:54-109): a threatening move continues a
        // chase only when the opponent's last move was an evasion; it breaks
        // the rule when the board with the mover simply set on dst is already
        // in the chase and dst is not the square the chaser last left
        evb = rec[R_ISF_EV];
        const bool ev_opp = (evb >> opp) & 1;
        if (threat && ev_opp) {
            uint64_t hs = h_before ^ zob(zt, src, p, ps) ^ zob(zt, dst, p, ps);
            if (attack) hs ^= zob(zt, dst, opp, pd);
            if (ring_has(hs) && !(chlast >= 0 && dst == chlast)) chv = 1;
            if (!ring_has(h)) ring_add(h);
            chlast = src;
        } else if (!threat) {
            chl = 0;
            chh = 0;
            chlast = -1;
            bloom = 0;
        }
        const uint32_t to = fld<uint32_t>(rec, R_ISF_THR + 4 * opp);
        const bool was_ev = (to & 0xFF) == (uint32_t)src || ((to >> 8) & 0xFF) == (uint32_t)src ||
                            ((to >> 16) & 0xFF) == (uint32_t)src || (to >> 24) == (uint32_t)src;
        evb = (uint8_t)((evb & ~(1u << p)) | ((was_ev ? 1u : 0u) << p));
    }

    // terminal caps (cu:383-395); the legal-move test is the caller's
    if (outcome == -1) {
        if (mn >= a.max_len) outcome = 2;
        else if (msa >= a.no_attack_limit) outcome = 2;
        else check_legal = true;
    }

    if (lane == 0) {
        rec[src] = ns;
        rec[dst] = nd;
        fld<uint64_t>(rec, R_ZHASH) = h;
        fld<int32_t>(rec, R_MSA) = msa;
        fld<int32_t>(rec, R_MOVENUM) = mn;
        fld<int16_t>(rec, R_HIST + 2 * head) = (int16_t)act;
        rec[R_HHEAD] = (uint8_t)((head + 1) & 31);
        rec[R_HLEN] = (uint8_t)min(hlen + 1, NHIST);
        fld<int8_t>(rec, R_PLAYER) = (int8_t)opp;
        if (!isf) {
            fld<int32_t>(rec, R_TSCOUNT + 4 * p) = tsc;
            fld<int16_t>(rec, R_TSLO + 2 * p) = (int16_t)tslo;
            fld<int16_t>(rec, R_TSHI + 2 * p) = (int16_t)tshi;
        } else {
            fld<uint32_t>(rec, R_ISF_THR + 4 * p) = thr;
            rec[R_ISF_EV] = evb;
            uint16_t* t = reinterpret_cast<uint16_t*>(tsq);
            if (!isf_keep_dst) {
                t[dst * 3] = (uint16_t)isf_new[0];
                t[dst * 3 + 1] = (uint16_t)isf_new[1];
                t[dst * 3 + 2] = (uint16_t)isf_new[2];
            }
            t[src * 3] = t[src * 3 + 1] = t[src * 3 + 2] = 0xFFFF;
        }
        rec[R_TSVIOL] = tsv;
        rec[R_CHHEAD + p] = (uint8_t)chh;
        rec[R_CHLEN + p] = (uint8_t)chl;
        fld<int8_t>(rec, R_CHLAST + p) = (int8_t)chlast;
        fld<uint64_t>(rec, R_BLOOM + 8 * p) = bloom;
        rec[R_CHVIOL] = chv;
        fld<int8_t>(rec, R_OUTCOME) = outcome;
        rec[R_TERM] = outcome != -1;
        if (flag_taken) rec[R_FLAGCAP] = 1;
        fld<int32_t>(rec, R_PROPPLY) = -1;
    }
    __syncwarp();
    return true;
}

// ---------------------------------------------------------------------------
// Observations, written straight from registers
// ---------------------------------------------------------------------------
//
// Stores cover whole rows wherever the values are dense: one warp store per
// infostate plane row (25 lanes x 4 elements) and 16-byte chunks for the u8
// mask.  Scalar 1- or 2-byte stores cost one L2 request each, so they are
// kept to the sparse one-hots (about 100 per env).

template <typename T>
struct IV;
template <>
struct IV<float> {
    static __device__ __forceinline__ float from(float f) { return f; }
};
template <>
struct IV<uint16_t> {
    static __device__ __forceinline__ uint16_t from(float f) { return __bfloat16_as_ushort(__float2bfloat16_rn(f)); }
};

template <typename T>
union Chunk {
    uint4 v;
    T e[16 / sizeof(T)];
};

__device__ __forceinline__ void st16(void* p, uint4 v) { *reinterpret_cast<uint4*>(p) = v; }
// Output stores of the global outputs.  kStream (the single-ply production
// step, whose every output line is written whole within a short window):
// st.global.cs, evict-first in L2, so finished output lines leave L2 ahead of
// the game records; measured 3% faster per config-2 step, and 11% slower for
// the Gumbel step kernel of config 3, which keeps plain stores.
template <bool kStream>
__device__ __forceinline__ void st_out(uint4* p, uint4 v) {
    if constexpr (kStream) __stcs(p, v);
    else *p = v;
}
template <bool kStream>
__device__ __forceinline__ void st_out(uint2* p, uint2 v) {
    if constexpr (kStream) __stcs(p, v);
    else *p = v;
}

template <typename T>
struct InfoGeom {
    static constexpr int PB = NSQ * (int)sizeof(T);          // bytes per plane
    static constexpr int R1B = ((43 * PB + 15) / 16) * 16;   // channels 0-42, padded
    static constexpr int HB = 32 * PB;                        // channels 456-487
};

// Four consecutive elements of one plane row (one lane's squares 4L..4L+3):
// two words of bf16 bits or four words of f32 bits.
template <typename T>
struct Quad;
template <>
struct Quad<uint16_t> {
    using V = uint2;
    // element pattern `pat` where mask byte j is 0xFF, 0 elsewhere
    static __device__ __forceinline__ V sel(uint32_t m, uint32_t pat) {
        const uint32_t p2 = pat | (pat << 16);
        return make_uint2(__byte_perm(m, 0, 0x1100) & p2, __byte_perm(m, 0, 0x3322) & p2);
    }
    static __device__ __forceinline__ V splat(uint32_t pat) {
        const uint32_t p2 = pat | (pat << 16);
        return make_uint2(p2, p2);
    }
    static __device__ __forceinline__ V orv(V a, V b) { return make_uint2(a.x | b.x, a.y | b.y); }
    // element pattern `pat` where byte j of m is 1, 0 where it is 0
    static __device__ __forceinline__ V ones(uint32_t m, uint32_t pat) {
        return make_uint2(__byte_perm(m, 0, 0x4140) * pat, __byte_perm(m, 0, 0x4342) * pat);
    }
    template <bool S>
    static __device__ __forceinline__ void st(uint8_t* p, V v) { st_out<S>(reinterpret_cast<uint2*>(p), v); }
    static __device__ __forceinline__ uint32_t bits(uint16_t v) { return v; }
};
template <>
struct Quad<float> {
    using V = uint4;
    static __device__ __forceinline__ V sel(uint32_t m, uint32_t pat) {
        return make_uint4(__byte_perm(m, 0, 0x0000) & pat, __byte_perm(m, 0, 0x1111) & pat,
                          __byte_perm(m, 0, 0x2222) & pat, __byte_perm(m, 0, 0x3333) & pat);
    }
    static __device__ __forceinline__ V splat(uint32_t pat) { return make_uint4(pat, pat, pat, pat); }
    static __device__ __forceinline__ V orv(V a, V b) { return make_uint4(a.x | b.x, a.y | b.y, a.z | b.z, a.w | b.w); }
    static __device__ __forceinline__ V ones(uint32_t m, uint32_t pat) {
        return make_uint4((m & 0xFF) * pat, ((m >> 8) & 0xFF) * pat, ((m >> 16) & 0xFF) * pat, (m >> 24) * pat);
    }
    template <bool S>
    static __device__ __forceinline__ void st(uint8_t* p, V v) { st_out<S>(reinterpret_cast<uint4*>(p), v); }
    static __device__ __forceinline__ uint32_t bits(float v) { return __float_as_uint(v); }
};

// Infostate of the side to move (stratego/env/infostate.py:37-109, channel
// meaning as csrc/stratego_buffer.cu:707-767).  Lanes 0..24 own squares
// 4L..4L+3: each derives its squares' features as byte vectors and writes
// its 4-element slice of every plane row, so one warp store covers a whole
// 100-element row.  The dense planes (12-42) are computed in full with byte
// SIMD compares; the sparse ones (0-11: one 1 per own piece; 456-487: one +1
// and one -1 per move) are zero rows plus one scalar store per non-zero.
// sd: the warp's 32-entry table of (src | dst << 8) of the last moves, most
// recent first.
// Per-square features of lane L's squares 4L..4L+3 as byte vectors.
struct SqFeat {
    uint32_t ot, ort, owt, fl;  // own type, opponent revealed type, own revealed type, flag bits
};
// Byte-parallel over the lane's 4 square codes: each field is a byte mask.
__device__ __forceinline__ SqFeat square_features(const uint8_t* rec, int lane) {
    constexpr uint32_t B1 = 0x01010101u;
    const uint32_t prep = rec[R_PLAYER] ? B1 : 0u;
    const uint32_t codes = *reinterpret_cast<const uint32_t*>(rec + 4 * lane);
    const uint32_t occ = (codes >> 5) & B1, blue = (codes >> 4) & B1;
    const uint32_t rev = (codes >> 7) & B1, mov = (codes >> 6) & B1;
    const uint32_t own = occ & ~(blue ^ prep), opp = occ ^ own;  // 0/1 per byte
    const uint32_t pc = codes & 0x0F0F0F0Fu;
    SqFeat f;
    f.ot = pc & (own * 0xFFu);
    f.ort = pc & ((opp & rev) * 0xFFu);
    f.owt = pc & ((own & rev) * 0xFFu);
    f.fl = (own & ~rev) | ((opp & ~rev) << 1) | ((occ ^ B1) << 2) | ((own & mov) << 3) | ((opp & mov) << 4);
    return f;
}

// Dense planes 12-42 (lanes 0..24).  Planes 12-35 hold, per side, 1/12 on
// every hidden piece of that side in all 12 rows and 1 on a revealed piece in
// its type's row: each lane stores the hidden-piece background in all 24 rows
// (the same two words for 12 rows, no per-row arithmetic), then sets the few
// revealed squares of its 4 squares to 1 with scalar stores (same thread, so
// the later store wins).  Planes 36-40 are flag rows, 41-42 constants.
template <typename T, bool kStream>
__device__ void write_info_dense(const uint8_t* rec, const KArgs& a, int lane, uint8_t* g) {
    if (lane >= 25) return;
    using Q = Quad<T>;
    constexpr int PB = InfoGeom<T>::PB;
    const SqFeat f = square_features(rec, lane);
    const uint32_t ONE = Q::bits(IV<T>::from(1.0f));
    const uint32_t TW = Q::bits(IV<T>::from(__fdiv_rn(1.0f, 12.0f)));
    uint8_t* gl = g + lane * 4 * (int)sizeof(T);
    const typename Q::V hid_o = Q::ones((f.fl >> 1) & 0x01010101u, TW);  // opponent hidden
    const typename Q::V hid_w = Q::ones(f.fl & 0x01010101u, TW);         // own hidden
#pragma unroll
    for (int t = 0; t < 12; ++t) {
        Q::template st<kStream>(gl + (12 + t) * PB, hid_o);
        Q::template st<kStream>(gl + (24 + t) * PB, hid_w);
    }
    T* gl1 = reinterpret_cast<T*>(gl);
    const T one = IV<T>::from(1.0f);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t to = (f.ort >> (8 * j)) & 0xFF, tw = (f.owt >> (8 * j)) & 0xFF;
        if (to) gl1[(11 + to) * NSQ + j] = one;  // 12-23: opponent revealed, one-hot
        if (tw) gl1[(23 + tw) * NSQ + j] = one;  // 24-35: own pieces the opponent has seen
    }
    // 36 own hidden, 37 opponent hidden, 38 empty (lakes included), 39 own moved, 40 opponent moved
#pragma unroll
    for (int i = 0; i < 5; ++i) Q::template st<kStream>(gl + (36 + i) * PB, Q::ones((f.fl >> i) & 0x01010101u, ONE));
    // 41 / 42: the two fractions (exact float32 quotients)
    const int mn = fld<int32_t>(rec, R_MOVENUM), msa = fld<int32_t>(rec, R_MSA);
    Q::template st<kStream>(gl + 41 * PB,
                            Q::splat(Q::bits(IV<T>::from(a.max_len > 0 ? __fdiv_rn((float)mn, (float)a.max_len) : 0.0f))));
    Q::template st<kStream>(gl + 42 * PB,
          Q::splat(Q::bits(IV<T>::from(a.no_attack_limit > 0 ? __fdiv_rn((float)msa, (float)a.no_attack_limit) : 0.0f))));
}

// Sparse planes: 0-11 (one 1 per own piece) and 456-487 (the k-th most recent
// move's +1 at dst, -1 at src).  Planes 0-11 are written as whole rows (one
// byte compare per type); the history planes as zero rows -- unless a
// producer warp streamed those already (kHistZeroed) -- and then the history
// non-zeros on top, from the same warp right away.  Every line is thus
// written completely within a short window: patching lines written much
// earlier measured slower once the output stream keeps the L2 full (the
// earlier lines are no longer in L2 when the patch arrives).
// DENSE_ALL also zeroes planes 43-455.
template <typename T, bool kHistZeroed, bool kStream>
__device__ void write_info_sparse(const uint8_t* rec, int lane, uint8_t* g, int hist_off, bool all) {
    using Q = Quad<T>;
    constexpr int PB = InfoGeom<T>::PB;
    if (lane < 25) {
        uint8_t* gl = g + lane * 4 * (int)sizeof(T);
        const SqFeat f = square_features(rec, lane);
        const uint32_t ONE = Q::bits(IV<T>::from(1.0f));
#pragma unroll
        for (int t = 0; t < 12; ++t)
            Q::template st<kStream>(gl + t * PB, Q::ones(__vcmpeq4(f.ot, (uint32_t)(t + 1) * 0x01010101u) & 0x01010101u, ONE));
        if (!kHistZeroed) {
            const typename Q::V Z = Q::splat(0u);
#pragma unroll 8
            for (int k = 0; k < 32; ++k) Q::template st<kStream>(gl + hist_off + k * PB, Z);
        }
    }
    __syncwarp();
    const int hl = rec[R_HLEN], hh = rec[R_HHEAD];
    if (lane < hl) {
        const int act = fld<int16_t>(rec, R_HIST + 2 * ((hh - 1 - lane) & 31));
        T* hs = reinterpret_cast<T*>(g + hist_off + lane * PB);
        hs[act % 100] = IV<T>::from(1.0f);
        hs[act / 100] = IV<T>::from(-1.0f);
    }
    if (all) {
        const uint4 Z = make_uint4(0, 0, 0, 0);
        for (int i = 43 * PB / 16 + lane; i < 456 * PB / 16; i += 32) st_out<kStream>(reinterpret_cast<uint4*>(g + i * 16), Z);
    }
}

// The zero rows of one env's history planes (456-487), streamed by the TMA
// engine as one bulk copy from the CTA's zero buffer (no multicast); issued
// by the producer lane.
template <typename T>
__device__ void bulk_zero_history(const uint8_t* zb, uint8_t* ginfo, int hist_off) {
    bulk_s2g(ginfo + hist_off, zb, 32 * InfoGeom<T>::PB);
}

// Legal mask (csrc/stratego_buffer.cu:448-507) of the side to move, built
// bit-packed in shared memory from the rays (bit j of byte k = flat action
// 8k+j), then written as bit-packed rows and / or expanded to u8 rows in
// whole 16-byte chunks.  Lane i takes the i-th square with moves (ascending;
// a second round above 32) and ORs in its piece's whole destination set at
// once: the row run [sq-left, sq+right] and the column comb sq-10*up ..
// sq+10*down (stride 10), less sq itself, as one 128-bit value placed at bit
// sq*100 (its first word is word sq*100/32; adjacent squares can share a
// word, hence the atomics).
__device__ void build_mask_bits(const uint16_t* rays, int lane, uint32_t* w) {
    using u128 = unsigned __int128;
    // bits 0, 10, 20, ..., 120
    constexpr uint64_t COMB_LO = 0x1004010040100401ull, COMB_HI = 0x0100401004010040ull;
    for (int i = lane; i < 79; i += 32) reinterpret_cast<uint4*>(w)[i] = make_uint4(0, 0, 0, 0);
    uint32_t has[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int sq = lane + 32 * k;
        has[k] = __ballot_sync(FULL, sq < NSQ && rays[sq] != 0);
    }
    __syncwarp();
    const int c0 = __popc(has[0]), c01 = c0 + __popc(has[1]), c012 = c01 + __popc(has[2]);
    const int np = c012 + __popc(has[3]);
#pragma unroll 1
    for (int base = 0; base < np; base += 32) {
        const int i = base + lane;
        if (i < np) {
            const int wi = i < c0 ? 0 : (i < c01 ? 1 : (i < c012 ? 2 : 3));
            const int k = i - (wi == 0 ? 0 : (wi == 1 ? c0 : (wi == 2 ? c01 : c012)));
            const uint32_t m = wi == 0 ? has[0] : (wi == 1 ? has[1] : (wi == 2 ? has[2] : has[3]));
            const int sq = 32 * wi + nth_bit(m, k);
            const uint32_t r = rays[sq];
            const int up = r & 15, left = (r >> 4) & 15, right = (r >> 8) & 15, down = r >> 12;
            const int f0 = sq * 100, b = f0 & 31;
            const int p = b + sq;  // bit of the piece's own square (never set)
            const u128 one = 1;
            const u128 run = (u128)((1u << (left + right + 1)) - 1u) << (p - left);
            const u128 comb = ((((u128)COMB_HI) << 64) | COMB_LO) & ((one << (10 * (up + down) + 1)) - 1);
            const u128 x = (run | (comb << (p - 10 * up))) & ~(one << p);
            uint32_t* wq = w + (f0 >> 5);
            atomicOr(wq, (uint32_t)x);
            atomicOr(wq + 1, (uint32_t)(x >> 32));
            atomicOr(wq + 2, (uint32_t)(x >> 64));
            atomicOr(wq + 3, (uint32_t)(x >> 96));
        }
    }
    __syncwarp();
}

__device__ __forceinline__ uint32_t nibble_bytes(uint32_t n) { return (n * 0x00204081u) & 0x01010101u; }

template <bool kStream>
__device__ void write_mask_u8(const uint32_t* w, int lane, uint8_t* g) {
    const uint16_t* b16 = reinterpret_cast<const uint16_t*>(w);
    for (int c = lane; c < NACT / 16; c += 32) {
        const uint32_t b = b16[c];
        st_out<kStream>(reinterpret_cast<uint4*>(g + c * 16),
                        make_uint4(nibble_bytes(b & 15), nibble_bytes((b >> 4) & 15), nibble_bytes((b >> 8) & 15),
                                   nibble_bytes(b >> 12)));
    }
}

// One bit-packed row (1250 bytes, 2-byte aligned: rows of consecutive envs
// are 1250 bytes apart): the 16-byte-aligned middle as 16-byte stores, read
// from shared memory at the row's 2-byte phase with funnel shifts; the
// partial chunks at either end as 2-byte stores.
__device__ void write_mask_bits(const uint32_t* w, int lane, uint8_t* g) {
    const int a = (int)(reinterpret_cast<uintptr_t>(g) & 15);  // even
    const int head = (16 - a) & 15;                             // bytes before the first aligned chunk
    const int nfull = (SB_MASK_BITS_BYTES - head) >> 4;
    const int tail = head + 16 * nfull;
    const uint16_t* s16 = reinterpret_cast<const uint16_t*>(w);
    uint16_t* g16 = reinterpret_cast<uint16_t*>(g);
    if (lane < head / 2) g16[lane] = s16[lane];
    if (lane < (SB_MASK_BITS_BYTES - tail) / 2) g16[tail / 2 + lane] = s16[tail / 2 + lane];
    const int sh = (head & 3) * 8;  // 0 or 16
    for (int c = lane; c < nfull; c += 32) {
        const int o = head + 16 * c;
        const uint32_t* q = w + (o >> 2);  // q[4] lies inside the 1264-byte bit buffer
        const uint32_t v0 = q[0], v1 = q[1], v2 = q[2], v3 = q[3], v4 = q[4];
        st16(g + o, make_uint4(__funnelshift_r(v0, v1, sh), __funnelshift_r(v1, v2, sh), __funnelshift_r(v2, v3, sh),
                               __funnelshift_r(v3, v4, sh)));
    }
}

// ---------------------------------------------------------------------------
// Debug build: bounds checks of a game record
// ---------------------------------------------------------------------------
//
// Built with -DSB_DEBUG_BOUNDS (libstratego_b200_debug.so), every kernel that
// plays or observes a game first checks that the record holds nothing the
// kernels would use as an out-of-range index: piece codes (they index the
// Zobrist table), the side to move, the history ring's head / length and its
// live entries (square indices of the history planes), the chase rings'
// heads / lengths, the two-square pair squares and the cached proposal.  A
// record that fails is left untouched and its game skipped for the launch,
// and SB_STATUS_BAD_STATE is raised; nothing traps.  Records written only by
// these kernels always pass; the checks are for records a caller loaded.
#ifdef SB_DEBUG_BOUNDS
constexpr bool kDebugBounds = true;
#else
constexpr bool kDebugBounds = false;
#endif

__device__ bool record_ok(const uint8_t* rec, int lane, int rules) {
    bool ok = true;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int sq = lane + 32 * k;
        if (sq < NSQ) {
            const uint8_t c = rec[sq];
            const int pc = c & C_PIECE;
            ok &= (c & C_OCC) ? (pc >= 1 && pc <= 12) : (c & (C_PIECE | C_BLUE)) == 0;
        }
    }
    const int hh = rec[R_HHEAD], hl = rec[R_HLEN];
    if (lane < hl && hl <= NHIST) {
        const int act = fld<int16_t>(rec, R_HIST + 2 * ((hh - 1 - lane) & 31));
        ok &= act >= 0 && act < NACT;
    }
    if (lane == 0) {
        const int p = fld<int8_t>(rec, R_PLAYER), oc = fld<int8_t>(rec, R_OUTCOME);
        ok &= (p == 0 || p == 1) && oc >= -1 && oc <= 2 && rec[R_TERM] <= 1;
        ok &= hh < NHIST && hl <= NHIST;
        for (int q = 0; q < 2; ++q) {
            ok &= rec[R_CHHEAD + q] < NRING && rec[R_CHLEN + q] <= NRING;
            const int last = fld<int8_t>(rec, R_CHLAST + q);
            ok &= last >= -1 && last < NSQ;
            if (rules == SB_RULES_CUDA) {
                const int lo = fld<int16_t>(rec, R_TSLO + 2 * q), hi = fld<int16_t>(rec, R_TSHI + 2 * q);
                ok &= lo >= -1 && lo < NSQ && hi >= -1 && hi < NSQ;
            }
        }
        const int prop = fld<int16_t>(rec, R_PROP);
        ok &= prop >= -1 && prop < NACT;
    }
    return __all_sync(FULL, ok);
}

// ---------------------------------------------------------------------------
// The per-env kernel
// ---------------------------------------------------------------------------

// MODE: MODE_GENERIC takes every decision from a.flags; the step modes fix
// apply + step + propose (and the policy) at compile time so that the hot
// kernel carries only the code it runs.
constexpr int MODE_GENERIC = 0, MODE_STEP_UNIFORM = 1, MODE_STEP_GUMBEL = 2, MODE_STEP_PROD = 3;
// added to a step mode: the kernel also carries the ISF repetition rules
// (the generic kernel always does; the CUDA-rules step kernels never pay for them)
constexpr int MODE_ISF = 8;
// added to MODE_STEP_PROD: a persistent step server that runs one ply per
// step the host publishes in mapped memory, until told to stop
constexpr int MODE_SERVE = 16;

// Step server handshake.  CTA 0 relays the host's step (polled over PCIe,
// bounded) into device memory; every CTA's thread 0 then waits (bounded) on
// that relay in L2, so PCIe carries one poller.  Returns 1 to run step t, 0
// to stop (asked to, or gave up).
__device__ int serve_wait(const KArgs& a, int64_t t) {
    const uint64_t t0 = global_ns();
    if (blockIdx.x == 0) {
        for (;;) {
            int64_t go;
            asm volatile("ld.acquire.sys.global.s64 %0, [%1];" : "=l"(go) : "l"(a.serve_ctl + SERVE_GO) : "memory");
            if (go >= t) {
                int64_t stop;
                asm volatile("ld.acquire.sys.global.s64 %0, [%1];" : "=l"(stop) : "l"(a.serve_ctl + SERVE_STOP) : "memory");
                asm volatile("st.relaxed.gpu.global.s64 [%0], %1;" ::"l"(a.serve_dev + SERVE_STOP), "l"(stop) : "memory");
                asm volatile("st.release.gpu.global.s64 [%0], %1;" ::"l"(a.serve_dev + SERVE_GO), "l"(t) : "memory");
                return stop ? 0 : 1;
            }
            if (global_ns() - t0 > (uint64_t)a.serve_limit_ns) break;
            __nanosleep(100);
        }
    } else {
        for (;;) {
            int64_t go;
            asm volatile("ld.acquire.gpu.global.s64 %0, [%1];" : "=l"(go) : "l"(a.serve_dev + SERVE_GO) : "memory");
            if (go >= t) {
                int64_t stop;
                asm volatile("ld.relaxed.gpu.global.s64 %0, [%1];" : "=l"(stop) : "l"(a.serve_dev + SERVE_STOP) : "memory");
                return stop ? 0 : 1;
            }
            if (global_ns() - t0 > (uint64_t)a.serve_limit_ns) break;
            __nanosleep(100);
        }
    }
    if (a.status) atomicOr(a.status, SB_STATUS_WAIT_TIMEOUT);
    return 0;
}

template <typename T, int MODE>
__global__ void __launch_bounds__(WARPS * 32, 4) env_kernel(const __grid_constant__ KArgs a) {
    constexpr int M = MODE & ~(MODE_ISF | MODE_SERVE);
    constexpr bool kServe = (MODE & MODE_SERVE) != 0;
    constexpr bool kStep = M != MODE_GENERIC;
    constexpr bool kProd = M == MODE_STEP_PROD;
    const bool isf_on = (M == MODE_GENERIC || (MODE & MODE_ISF) != 0) && a.rules == SB_RULES_ISF;
    constexpr int kPol = (M == MODE_STEP_UNIFORM || kProd) ? SB_POLICY_UNIFORM
                         : (M == MODE_STEP_GUMBEL ? SB_POLICY_GUMBEL : -1);
    auto has = [&](uint32_t f) -> bool {
        if (kStep) {
            if (f & (F_RESET_PLANES | F_RESET_POOL | F_SAMPLE_OUT | F_HAS_LEGAL)) return false;
            if (f & F_PROPOSE) return true;
            if (f & (F_APPLY | F_STEP)) return a.n_plies > 0;
        }
        return (a.flags & f) != 0;
    };
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(16) int64_t s_zob[ZOB_N];
    // s_bar[0]: the Zobrist table has landed.  MODE_STEP_PROD only: [1] the
    // producer's zero rows of a batch are complete, [2] every env warp has
    // seen [1] for that batch (the producer then starts the next batch).
    __shared__ __align__(8) uint64_t s_bar[3];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    constexpr int ENVW = kProd ? WARPS - 1 : WARPS;  // warps that play envs
    const bool producer = kProd && w == WARPS - 1;
    uint8_t* zb = smem;  // MODE_STEP_PROD: the zero buffer precedes the warps' regions
    uint8_t* ws = smem + (kProd ? ZERO_BYTES : 0) + w * a.sm_warp;
    if (threadIdx.x == 0) {
        mbar_init(&s_bar[0], 1);
        mbar_init(&s_bar[1], 1);
        mbar_init(&s_bar[2], ENVW);
        mbar_fence_init();
    }
    __syncthreads();
    if (producer) {
        for (int i = lane; i < ZERO_BYTES / 16; i += 32) st16(zb + i * 16, make_uint4(0, 0, 0, 0));
        fence_async_smem();
        __syncwarp();
    }
    // Programmatic dependent launch (host side: launch_mode).  The next
    // launch on the stream may start its own prologue now, on SMs this launch
    // leaves; this launch waits here until the launch before it has completed
    // and its writes are visible, before touching global memory.  Both are
    // no-ops for a launch made without the attribute.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    // The Zobrist table lives in shared memory, so the game logic never waits
    // on HBM for it while the outputs stream out.  One bulk copy brings it in
    // while the warps load their records; a warp waits for it only before
    // its first lookup.
    if (threadIdx.x == 0) {
        mbar_arrive_expect_tx(&s_bar[0], ZOB_N * 8);
        bulk_g2s(s_zob, a.zob, ZOB_N * 8, &s_bar[0]);
    }
    bool zob_ready = false;
    auto zob_wait = [&]() {
        if (!zob_ready) {
            if (!mbar_wait(&s_bar[0], 0) && lane == 0 && a.status) atomicOr(a.status, SB_STATUS_WAIT_TIMEOUT);
            zob_ready = true;
        }
    };
    uint8_t* rec = ws;
    uint16_t* rays = reinterpret_cast<uint16_t*>(ws + SM_RAYS);
    uint16_t* scratch = reinterpret_cast<uint16_t*>(ws + SM_SCRATCH);
    uint32_t* wbits = reinterpret_cast<uint32_t*>(ws + SM_BITS);
    constexpr int PB = InfoGeom<T>::PB;
    const bool compact = a.info_layout == SB_LAYOUT_COMPACT;
    const int64_t info_env = (int64_t)(compact ? 76 : NCH) * PB;
    const int hist_off = (compact ? 44 : 456) * PB;
    // MODE_STEP_PROD is single-ply: one batch of envs per iteration
    const int np = (kStep && !kProd && a.n_plies > 1) ? a.n_plies : 1;
    const bool zeros = kProd && has(F_INFO);  // the producer streams the history planes' zero rows
    const int64_t stride = (int64_t)gridDim.x * ENVW;
    const int64_t first = (int64_t)blockIdx.x * ENVW;
    int64_t iter = 0;
    // step server: the CTA's actions cross PCIe as one coalesced read; the
    // step's results go back as one copy by the CTA that completes the step
    __shared__ int s_cmd, s_last;
    __shared__ int64_t s_act[WARPS];
    for (int64_t t = 1;; ++t) {
      if (kServe) {
        if (threadIdx.x == 0) s_cmd = serve_wait(a, t);
        __syncthreads();
        if (s_cmd != 1) break;
        if (a.actions && producer && lane < ENVW && first + lane < a.n)
            s_act[lane] = (int64_t)__ldcv(reinterpret_cast<const long long*>(a.actions) + first + lane);
        __syncthreads();
      }
      const int64_t ply_base = kServe ? a.ply + t - 1 : a.ply;
      for (int64_t base = first; base < a.n; base += stride) {
        if (producer) {
            if (zeros) {
                // at most one batch ahead of the slowest env warp
                if (iter > 0 && !mbar_wait(&s_bar[2], (uint32_t)((iter - 1) & 1)) && lane == 0 && a.status)
                    atomicOr(a.status, SB_STATUS_WAIT_TIMEOUT);
                if (lane == 0) {
                    const int64_t s_next = has(F_APPLY) ? (a.slot0 + 1 == a.n_slots ? 0 : a.slot0 + 1) : a.slot0;
                    for (int j = 0; j < ENVW && base + j < a.n; ++j) {
                        const int64_t in = s_next * a.n + base + j;
                        bulk_zero_history<T>(zb, reinterpret_cast<uint8_t*>(a.info) + in * info_env, hist_off);
                    }
                    bulk_commit();
                    bulk_wait_all();
                    // the zero rows are written before anything stored on top
                    fence_async_global();
                    mbar_arrive(&s_bar[1]);
                }
                __syncwarp();
            }
            ++iter;
            continue;
        }
        const int64_t e = base + w;
        bool live = e < a.n;
        if (live) {
            reinterpret_cast<uint2*>(rec)[lane] = reinterpret_cast<const uint2*>(a.rec + e * REC)[lane];
            __syncwarp();
        }
        int64_t* ring2 = a.ring + e * 2 * NRING;
        bool dirty = false;
        bool rays_ok = false;  // rays / n_moves describe the side to move of the current board
        int n_moves = 0;

        if (live && (has(F_RESET_PLANES) || has(F_RESET_POOL)) && (has(F_FORCE) || rec[R_TERM])) {
            zob_wait();
            reset_env(rec, ring2, a, s_zob, e, has(F_RESET_POOL), lane, isf_on);
            dirty = true;
        }
        if (kDebugBounds && live && !record_ok(rec, lane, a.rules)) {
            // the game is skipped: its record and outputs stay as they are
            if (lane == 0 && a.status) atomicOr(a.status, SB_STATUS_BAD_STATE);
            live = false;
            dirty = false;
        }

        // ring slots of the ply's transition (s_cur) and of its new state (s_next)
        int32_t s_cur = a.slot0, s_nx = a.slot0;
        for (int p = 0; p < np; ++p, ++iter, s_cur = s_nx) {
            // outside MODE_STEP_PROD the CTA's warps start each ply together:
            // they then run the same code and write neighbouring envs' rows
            // at about the same time (measured faster than letting them drift)
            if (!kProd) __syncthreads();
            const int64_t ply = ply_base + p;
            s_nx = has(F_APPLY) ? (s_cur + 1 == a.n_slots ? 0 : s_cur + 1) : a.slot0;
            const int32_t s_next = s_nx;
            const int64_t ic = (int64_t)s_cur * a.n + e, in = (int64_t)s_next * a.n + e;
            uint8_t* ginfo = has(F_INFO) ? reinterpret_cast<uint8_t*>(a.info) + in * info_env : nullptr;
            // the uniform proposal's random word depends only on (seed, env,
            // ply): drawn first, off the game logic's critical path
            const int64_t pp = has(F_PROPOSE) ? (has(F_APPLY) ? ply + 1 : ply) : ply_base;
            uint32_t u_prop = 0;
            if (kPol == SB_POLICY_UNIFORM)
                u_prop = philox_rk((uint32_t)(a.env_base + e), (uint32_t)pp, (uint32_t)((uint64_t)pp >> 32), TAG_ACTION,
                                   a.rk).x;
          if (live) {
            struct {
                bool valid = false, term = false, ended = false;
                int8_t oc = -1;
                int64_t act = -1;
                float lp = 0.0f;
                int32_t len = 0;
            } tr;
            if (has(F_APPLY)) {
                const bool was_term = rec[R_TERM] != 0;
                int64_t act = -1;
                float lp = 0.0f;
                if (!was_term) {
                    const int pm = rec[R_PLAYER];
                    int n_legal = -1;
                    if (a.actions) act = kServe ? s_act[w] : a.actions[e];
                    if (!a.actions || has(F_STEP)) {
                        if (fld<int32_t>(rec, R_PROPPLY) == (int32_t)ply &&
                            rec[R_PROPKIND] == (kPol >= 0 ? kPol : a.policy) && !a.logits) {
                            n_legal = fld<int16_t>(rec, R_NLEGAL);
                            if (!a.actions) {
                                act = fld<int16_t>(rec, R_PROP);
                                lp = fld<float>(rec, R_PROPLP);
                            }
                        } else {
                            n_legal = enumerate(rec, pm, rays, lane);
                            if (!a.actions) {
                                int ac;
                                choose_cold<kPol>(a.rk, a.env_base, a.logits, a.policy, rays, n_legal, e, ply, lane, ac,
                                                  lp, scratch);
                                act = ac;
                            }
                        }
                    }
                    if (has(F_STEP) && n_legal == 0) {
                        // a start position whose side to move cannot move: it
                        // loses (the rule of stratego/env/rules.py:406-413)
                        if (lane == 0) {
                            fld<int8_t>(rec, R_OUTCOME) = (int8_t)(pm == 0 ? 1 : 0);
                            rec[R_TERM] = 1;
                            fld<int32_t>(rec, R_PROPPLY) = -1;
                        }
                        act = -1;
                        __syncwarp();
                    } else {
                        bool chk, flag;
                        zob_wait();
                        const bool ok = apply_env(rec, ring2, a, s_zob, act, lane, chk, flag,
                                                  isf_on ? a.isf + e * ISF_TS_BYTES : nullptr);
                        if (ok) rays_ok = false;  // the board changed
                        if (!ok) {
                            if (lane == 0) fld<int32_t>(rec, R_INVALID) += 1;
                            __syncwarp();
                        } else if (chk) {
                            n_moves = enumerate(rec, rec[R_PLAYER], rays, lane);
                            rays_ok = true;
                            if (n_moves == 0) {
                                if (lane == 0) {
                                    fld<int8_t>(rec, R_OUTCOME) = (int8_t)(rec[R_PLAYER] == 0 ? 1 : 0);
                                    rec[R_TERM] = 1;
                                }
                                __syncwarp();
                            }
                        }
                    }
                }
                const bool term = rec[R_TERM] != 0;
                if (lane == 0 && term) fld<int32_t>(rec, R_TSINCE) += 1;
                // the transition's outputs are stored at the end of the ply, so
                // the game logic never waits behind the output stream
                tr.valid = true;
                tr.oc = fld<int8_t>(rec, R_OUTCOME);
                tr.term = term;
                tr.ended = term && !was_term;
                tr.act = act;
                tr.lp = lp;
                tr.len = fld<int32_t>(rec, R_MOVENUM);
                __syncwarp();
                dirty = true;
                if (has(F_AUTO_RESET) && term) {
                    zob_wait();
                    reset_env(rec, ring2, a, s_zob, e, true, lane, isf_on);
                    rays_ok = false;
                }
            }

            const bool observe = has(F_MASK_U8) || has(F_MASK_BITS) || has(F_PROPOSE) || has(F_HAS_LEGAL) ||
                                 has(F_SAMPLE_OUT);
            int n = 0;
            if (observe) {
                if (!rays_ok) n_moves = enumerate(rec, rec[R_PLAYER], rays, lane);
                n = n_moves;
            }
            if (has(F_PROPOSE) || has(F_SAMPLE_OUT)) {
                int ac;
                float lp;
                // a game that is over (and was not reset) proposes no move: -1, log-prob 0
                const int n_pick = has(F_PROPOSE) && rec[R_TERM] ? 0 : n;
                choose<kPol>(Pick{a.rk, a.env_base, a.logits, a.policy}, rays, n_pick, e, pp, lane, ac, lp, scratch,
                             kPol == SB_POLICY_UNIFORM ? &u_prop : nullptr);
                if (lane == 0) {
                    if (has(F_PROPOSE)) {
                        fld<int16_t>(rec, R_PROP) = (int16_t)ac;
                        fld<int32_t>(rec, R_PROPPLY) = a.logits ? -1 : (int32_t)pp;
                        rec[R_PROPKIND] = (uint8_t)(kPol >= 0 ? kPol : a.policy);
                        fld<int16_t>(rec, R_NLEGAL) = (int16_t)n_pick;
                        fld<float>(rec, R_PROPLP) = lp;
                        if (a.next_action) a.next_action[in] = (int16_t)ac;
                        if (a.next_logprob) a.next_logprob[in] = lp;
                    }
                    if (has(F_SAMPLE_OUT)) {
                        if (a.sampled) a.sampled[e] = ac;
                        if (a.sampled_lp) a.sampled_lp[e] = lp;
                    }
                }
                if (has(F_PROPOSE)) dirty = true;
            }
            if (lane == 0) {
                if (has(F_HAS_LEGAL)) a.has_legal[e] = n > 0;
                if (has(F_HASH)) a.hash[in] = fld<int64_t>(rec, R_ZHASH);
                if (tr.valid) {
                    if (a.reward) a.reward[ic] = tr.oc == 0 ? 1.0f : (tr.oc == 1 ? -1.0f : 0.0f);
                    if (a.done) a.done[ic] = tr.term ? 1 : 0;
                    if (a.action_taken) a.action_taken[ic] = tr.act;
                    if (a.logprob_taken) a.logprob_taken[ic] = tr.lp;
                    if (a.stats && tr.ended) {
                        atomicAdd(reinterpret_cast<unsigned long long*>(&a.stats[0]), 1ull);
                        atomicAdd(reinterpret_cast<unsigned long long*>(&a.stats[tr.oc == 0 ? 1 : (tr.oc == 1 ? 2 : 3)]),
                                  1ull);
                        atomicAdd(reinterpret_cast<unsigned long long*>(&a.stats[4]), (unsigned long long)tr.len);
                    }
                }
            }
            __syncwarp();
            // outputs of the new state.  Dense rows need no zero pass.  In
            // MODE_STEP_PROD the odd warps write them last, so that their
            // stream overlaps the even warps' sparse and mask rows and the
            // other way round.
            if (has(F_INFO) && !(zeros && (w & 1))) write_info_dense<T, kProd>(rec, a, lane, ginfo);
          }
            if (zeros) {
                // this batch's zero rows are complete (producer)
                if (!mbar_wait(&s_bar[1], (uint32_t)(iter & 1)) && lane == 0 && a.status)
                    atomicOr(a.status, SB_STATUS_WAIT_TIMEOUT);
                __syncwarp();
                if (lane == 0) mbar_arrive(&s_bar[2]);
            }
          if (live) {
            const bool all = a.info_layout == SB_LAYOUT_DENSE_ALL;
            if (has(F_INFO)) write_info_sparse<T, kProd, kProd>(rec, lane, ginfo, hist_off, all);
            if (has(F_MASK_U8) || has(F_MASK_BITS)) {
                build_mask_bits(rays, lane, wbits);
                if (has(F_MASK_U8)) write_mask_u8<kProd>(wbits, lane, a.mask_u8 + in * NACT);
                if (has(F_MASK_BITS)) write_mask_bits(wbits, lane, a.mask_bits + in * SB_MASK_BITS_BYTES);
            }
            if (zeros && (w & 1) && has(F_INFO)) write_info_dense<T, kProd>(rec, a, lane, ginfo);
            __syncwarp();
          }
        }

        if (live && dirty) reinterpret_cast<uint2*>(a.rec + e * REC)[lane] = reinterpret_cast<const uint2*>(rec)[lane];
        __syncwarp();
      }
      if (!kServe) break;
      // count the CTA in; the one that completes the step copies the result
      // block to page-locked host memory and tells the host
      __syncthreads();
      if (threadIdx.x == 0) {
          unsigned long long old;
          asm volatile("atom.acq_rel.gpu.global.add.u64 %0, [%1], 1;"
                       : "=l"(old)
                       : "l"(a.serve_dev + DEV_DONE_COUNT)
                       : "memory");
          s_last = (int64_t)old + 1 == (int64_t)gridDim.x * t;
      }
      __syncthreads();
      if (s_last) {
          const uint4* src = reinterpret_cast<const uint4*>(a.serve_back_dev);
          uint4* dst = reinterpret_cast<uint4*>(a.serve_back_host);
          for (int64_t i = threadIdx.x; i < a.serve_back_bytes / 16; i += blockDim.x) dst[i] = __ldcg(src + i);
          __threadfence_system();
      }
      __syncthreads();
      if (threadIdx.x == 0 && s_last)
          asm volatile("st.release.sys.global.s64 [%0], %1;" ::"l"(a.serve_ctl + SERVE_DONE), "l"(t) : "memory");
    }
    // the table's bulk copy must land before the CTA's shared memory goes away
    if (threadIdx.x == 0) zob_wait();
}

// ---------------------------------------------------------------------------
// Belief resampling for search (north-star; no reference kernel)
// ---------------------------------------------------------------------------
//
// Sample env e starts as a copy of root r = root_of[e] whose opponent (the
// side not to move) has its unrevealed pieces' identities re-dealt: the
// moved unrevealed squares first draw, without replacement, from the movable
// identities of that multiset (a moved piece is never a Bomb or the Flag),
// then the remaining identities are shuffled over the unmoved unrevealed
// squares.  Both draws are uniform, so the deal is uniform over the
// assignments consistent with what the side to move has seen.  Philox key:
// the samples' seed; counter: (global sample index, block, TAG_BELIEF).
// The copy keeps the board's flags, counters, history and two-square state;
// its chase rings start empty (their hashes described the true identities)
// and its Zobrist hash is recomputed.
__global__ void __launch_bounds__(WARPS * 32) belief_kernel(const uint8_t* root_rec, int64_t n_roots,
                                                           const int64_t* root_of, const __grid_constant__ KArgs a,
                                                           const uint8_t* root_isf) {
    __shared__ __align__(16) uint8_t srec[WARPS][REC];
    // lane 0's Fisher-Yates lists: moved / unmoved hidden squares, the
    // identities (movable ones first), and the movable / immobile identities
    // as found; in shared memory, not in local memory
    __shared__ uint8_t s_fy[WARPS][5][40];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    uint8_t* rec = srec[w];
    const int64_t nwarps = (int64_t)gridDim.x * WARPS;
    for (int64_t e = (int64_t)blockIdx.x * WARPS + w; e < a.n; e += nwarps) {
        int64_t r = root_of[e];
        const bool bad = r < 0 || r >= n_roots;
        if (bad) r = 0;
        reinterpret_cast<uint2*>(rec)[lane] = reinterpret_cast<const uint2*>(root_rec + r * REC)[lane];
        if (a.rules == SB_RULES_ISF) {
            // the per-piece two-square state follows the squares, not the identities
            const uint2* src = reinterpret_cast<const uint2*>(root_isf + r * ISF_TS_BYTES);
            uint2* dst = reinterpret_cast<uint2*>(a.isf + e * ISF_TS_BYTES);
            for (int i = lane; i < ISF_TS_BYTES / 8; i += 32) dst[i] = src[i];
        }
        __syncwarp();
        if (kDebugBounds && !record_ok(rec, lane, a.rules)) {
            if (lane == 0 && a.status) atomicOr(a.status, SB_STATUS_BAD_STATE);
            continue;  // the sample is left as it was
        }
        const int opp = 1 - rec[R_PLAYER];
        unsigned hid[4], mov[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int sq = lane + 32 * k;
            const uint8_t c = sq < NSQ ? rec[sq] : 0;
            const bool h = (c & C_OCC) && ((c >> 4) & 1) == opp && !(c & C_REV);
            hid[k] = __ballot_sync(FULL, h);
            mov[k] = __ballot_sync(FULL, h && (c & C_MOVED));
        }
        if (lane == 0) {
            if (bad && a.status) atomicOr(a.status, SB_STATUS_BAD_SETUP);
            uint8_t *msq = s_fy[w][0], *usq = s_fy[w][1], *pcs = s_fy[w][2], *movp = s_fy[w][3], *immp = s_fy[w][4];
            int nm = 0, nu = 0, nmov = 0, nimm = 0;
            for (int k = 0; k < 4; ++k) {
                unsigned hb = hid[k];
                while (hb) {
                    const int b = __ffs(hb) - 1;
                    hb &= hb - 1;
                    const int sq = 32 * k + b;
                    const int pc = rec[sq] & C_PIECE;
                    if (nm + nu < 40) {
                        if ((mov[k] >> b) & 1) msq[nm++] = (uint8_t)sq;
                        else usq[nu++] = (uint8_t)sq;
                        if (can_move(pc)) movp[nmov++] = (uint8_t)pc;
                        else immp[nimm++] = (uint8_t)pc;
                    }
                }
            }
            // identities: movable ones first, then bombs / flag
            int np_ = 0;
            for (int i = 0; i < nmov; ++i) pcs[np_++] = movp[i];
            for (int i = 0; i < nimm; ++i) pcs[np_++] = immp[i];
            const int64_t ge = a.env_base + e;
            uint4 words = make_uint4(0, 0, 0, 0);
            int used = 4, blk = 0;
            auto draw = [&](uint32_t bound) -> int {
                if (used == 4) {
                    words = philox_rk((uint32_t)ge, (uint32_t)blk++, (uint32_t)((uint64_t)ge >> 32), TAG_BELIEF, a.rk);
                    used = 0;
                }
                const uint32_t wd = used == 0 ? words.x : (used == 1 ? words.y : (used == 2 ? words.z : words.w));
                ++used;
                return (int)mulshift(wd, bound);
            };
            // 1) moved squares draw from the movable identities (partial Fisher-Yates)
            const int take = nm < nmov ? nm : nmov;
            for (int i = 0; i < take; ++i) {
                const int j = i + draw((uint32_t)(nmov - i));
                const uint8_t t = pcs[i];
                pcs[i] = pcs[j];
                pcs[j] = t;
            }
            // 2) the rest shuffled over the unmoved squares (Fisher-Yates on the tail)
            for (int i = np_ - 1; i > take; --i) {
                const int j = take + draw((uint32_t)(i - take + 1));
                const uint8_t t = pcs[i];
                pcs[i] = pcs[j];
                pcs[j] = t;
            }
            for (int i = 0; i < nm; ++i) rec[msq[i]] = (uint8_t)((rec[msq[i]] & ~C_PIECE) | pcs[i]);
            for (int i = 0; i < nu; ++i) rec[usq[i]] = (uint8_t)((rec[usq[i]] & ~C_PIECE) | pcs[nm + i]);
            rec[R_CHHEAD] = rec[R_CHHEAD + 1] = 0;
            rec[R_CHLEN] = rec[R_CHLEN + 1] = 0;
            fld<int8_t>(rec, R_CHLAST) = -1;
            fld<int8_t>(rec, R_CHLAST + 1) = -1;
            fld<int32_t>(rec, R_PROPPLY) = -1;
            fld<int16_t>(rec, R_PROP) = -1;
            fld<uint64_t>(rec, R_BLOOM) = 0;
            fld<uint64_t>(rec, R_BLOOM + 8) = 0;
        }
        __syncwarp();
        uint64_t h = 0;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int sq = lane + 32 * k;
            if (sq < NSQ) {
                const uint8_t c = rec[sq];
                if (c & C_OCC) h ^= zob(a.zob, sq, (c >> 4) & 1, c & C_PIECE);
            }
        }
        h = warp_xor64(h);
        if (lane == 0) fld<uint64_t>(rec, R_ZHASH) = h;
        int4* rg = reinterpret_cast<int4*>(a.ring + e * 2 * NRING);
        rg[lane] = make_int4(0, 0, 0, 0);
        rg[lane + 32] = make_int4(0, 0, 0, 0);
        __syncwarp();
        reinterpret_cast<uint2*>(a.rec + e * REC)[lane] = reinterpret_cast<const uint2*>(rec)[lane];
        __syncwarp();
    }
}

// ---------------------------------------------------------------------------
// Small kernels
// ---------------------------------------------------------------------------

__global__ void hello_kernel(int32_t* out) {
    if (threadIdx.x == 0 && blockIdx.x == 0) out[0] = 42;
}

// Fresh-buffer state (csrc/stratego_buffer.cpp:24-55).
__global__ void init_kernel(uint8_t* rec, int64_t* ring, int64_t n, int32_t rules, uint8_t* isf) {
    const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= n) return;
    uint8_t* r = rec + e * REC;
    for (int i = 0; i < REC / 16; ++i) reinterpret_cast<int4*>(r)[i] = make_int4(0, 0, 0, 0);
    fld<int8_t>(r, R_OUTCOME) = -1;
    if (rules == SB_RULES_ISF) {
        fld<uint64_t>(r, R_ISF_THR) = ~0ull;
        fld<uint64_t>(r, R_ISF_EV) = ~0ull << 8;
        uint2* t = reinterpret_cast<uint2*>(isf + e * ISF_TS_BYTES);
        for (int i = 0; i < ISF_TS_BYTES / 8; ++i) t[i] = make_uint2(~0u, ~0u);
    } else {
        fld<int16_t>(r, R_TSLO) = -1;
        fld<int16_t>(r, R_TSLO + 2) = -1;
        fld<int16_t>(r, R_TSHI) = -1;
        fld<int16_t>(r, R_TSHI + 2) = -1;
    }
    fld<int8_t>(r, R_CHLAST) = -1;
    fld<int8_t>(r, R_CHLAST + 1) = -1;
    fld<int16_t>(r, R_PROP) = -1;
    fld<int32_t>(r, R_PROPPLY) = -1;
    int4* g = reinterpret_cast<int4*>(ring + e * 2 * NRING);
    for (int i = 0; i < 2 * NRING / 2; ++i) g[i] = make_int4(0, 0, 0, 0);
}

// Pool entry i: Fisher-Yates over the roster, Philox words (ctr: i_lo, block,
// i_hi, TAG_SETUP), j = (w * (i+1)) >> 32.
__global__ void pool_kernel(uint64_t seed, int64_t start, int64_t count, uint8_t* out) {
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= count) return;
    const uint64_t idx = (uint64_t)(start + t);
    uint8_t p[40];
    const uint8_t counts[13] = {0, 1, 8, 5, 4, 4, 4, 3, 2, 1, 1, 1, 6};
    int k = 0;
    for (int pt = 1; pt <= 12; ++pt)
        for (int j = 0; j < counts[pt]; ++j) p[k++] = (uint8_t)pt;
    for (int blk = 0; blk < 10; ++blk) {
        const uint4 w = philox((uint32_t)idx, (uint32_t)blk, (uint32_t)(idx >> 32), TAG_SETUP, seed);
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
        for (int q = 0; q < 4; ++q) {
            const int d = blk * 4 + q;
            if (d >= 39) break;
            const int i = 39 - d;
            const int j = (int)mulshift(ws[q], (uint32_t)(i + 1));
            const uint8_t tmp = p[i];
            p[i] = p[j];
            p[j] = tmp;
        }
    }
    for (int i = 0; i < 40; ++i) out[t * 40 + i] = p[i];
}

__global__ void export_kernel(const uint8_t* rec, int64_t n, sb_export o, int32_t rules, const uint8_t* isf) {
    const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= n) return;
    const uint8_t* r = rec + e * REC;
    for (int q = 0; q < NSQ; ++q) {
        const uint8_t c = r[q];
        if (o.board_owner) o.board_owner[e * NSQ + q] = (int8_t)owner_of(c);
        if (o.board_piece) o.board_piece[e * NSQ + q] = (int8_t)((c & C_OCC) ? (c & C_PIECE) : 0);
        if (o.moved_squares) o.moved_squares[e * NSQ + q] = (c & C_MOVED) ? 1 : 0;
        if (o.revealed_squares) o.revealed_squares[e * NSQ + q] = (c & C_REV) ? 1 : 0;
    }
    const int8_t oc = *reinterpret_cast<const int8_t*>(r + R_OUTCOME);
    if (o.current_player) o.current_player[e] = *reinterpret_cast<const int8_t*>(r + R_PLAYER);
    if (o.outcome) o.outcome[e] = oc;
    if (o.terminated) o.terminated[e] = r[R_TERM];
    if (o.flag_captured) o.flag_captured[e] = r[R_FLAGCAP];
    if (o.move_number) o.move_number[e] = *reinterpret_cast<const int32_t*>(r + R_MOVENUM);
    if (o.moves_since_attack) o.moves_since_attack[e] = *reinterpret_cast<const int32_t*>(r + R_MSA);
    if (o.terminated_since) o.terminated_since[e] = *reinterpret_cast<const int32_t*>(r + R_TSINCE);
    if (o.move_history)
        for (int i = 0; i < NHIST; ++i) o.move_history[e * NHIST + i] = *reinterpret_cast<const int16_t*>(r + R_HIST + 2 * i);
    if (o.move_history_head) o.move_history_head[e] = r[R_HHEAD];
    if (o.move_history_len) o.move_history_len[e] = r[R_HLEN];
    const bool is = rules == SB_RULES_ISF;  // the two rule sets share record bytes 120-135
    for (int p = 0; p < 2; ++p) {
        if (o.two_square_count) o.two_square_count[e * 2 + p] = is ? 0 : *reinterpret_cast<const int32_t*>(r + R_TSCOUNT + 4 * p);
        if (o.two_square_pair_lo) o.two_square_pair_lo[e * 2 + p] = is ? -1 : *reinterpret_cast<const int16_t*>(r + R_TSLO + 2 * p);
        if (o.two_square_pair_hi) o.two_square_pair_hi[e * 2 + p] = is ? -1 : *reinterpret_cast<const int16_t*>(r + R_TSHI + 2 * p);
        if (o.isf_evasion) o.isf_evasion[e * 2 + p] = is ? (r[R_ISF_EV] >> p) & 1 : 0;
        for (int k = 0; k < 4; ++k)
            if (o.isf_threats) o.isf_threats[e * 8 + p * 4 + k] = is ? *reinterpret_cast<const int8_t*>(r + R_ISF_THR + 4 * p + k) : -1;
        if (o.chase_hash_head) o.chase_hash_head[e * 2 + p] = r[R_CHHEAD + p];
        if (o.chase_hash_len) o.chase_hash_len[e * 2 + p] = r[R_CHLEN + p];
        if (o.chase_last_src) o.chase_last_src[e * 2 + p] = *reinterpret_cast<const int8_t*>(r + R_CHLAST + p);
    }
    if (o.two_square_violation) o.two_square_violation[e] = r[R_TSVIOL];
    if (o.chasing_violation) o.chasing_violation[e] = r[R_CHVIOL];
    if (o.episode) o.episode[e] = *reinterpret_cast<const int32_t*>(r + R_EPISODE);
    if (o.invalid_count) o.invalid_count[e] = *reinterpret_cast<const int32_t*>(r + R_INVALID);
    if (o.reward) o.reward[e] = oc == 0 ? 1.0f : (oc == 1 ? -1.0f : 0.0f);
    if (o.isf_two_square)
        for (int i = 0; i < ISF_TS_BYTES; ++i) o.isf_two_square[e * ISF_TS_BYTES + i] = is ? isf[e * ISF_TS_BYTES + i] : 0xFF;
}

__global__ void sum_move_kernel(const uint8_t* rec, int64_t n, int64_t* out) {
    int64_t acc = 0;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x)
        acc += *reinterpret_cast<const int32_t*>(rec + e * REC + R_MOVENUM);
    for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(FULL, acc, o);
    if ((threadIdx.x & 31) == 0 && acc) atomicAdd(reinterpret_cast<unsigned long long*>(out), (unsigned long long)acc);
}

}  // namespace sb

// ===========================================================================
// Host side: argument checks, launch configuration, C ABI
// ===========================================================================

// Staging array of sb_step_host_noalloc: the host actions are copied here,
// so its callers need not allocate device memory.  Host code must not use
// the symbol as a device address; it asks for the address once per device.
static __device__ __align__(256) int64_t g_noalloc_actions[SB_NOALLOC_MAX_ENVS];

namespace {

thread_local char g_err[512] = "";

int fail(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof g_err, fmt, ap);
    va_end(ap);
    return code;
}

int cuda_fail(cudaError_t e, const char* what) {
    return fail(SB_E_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

int check_state(const sb_state* s) {
    if (!s) return fail(SB_E_ARG, "state is NULL");
    if (s->n < 0) return fail(SB_E_ARG, "n < 0");
    if (s->n == 0) return SB_OK;
    if (!s->records || !s->chase_ring || !s->zobrist) return fail(SB_E_ARG, "records/chase_ring/zobrist is NULL");
    if (!aligned(s->records, 16) || !aligned(s->chase_ring, 16) || !aligned(s->zobrist, 16))
        return fail(SB_E_ARG, "records/chase_ring/zobrist not 16-byte aligned");
    if (s->rules != SB_RULES_CUDA && s->rules != SB_RULES_ISF) return fail(SB_E_ARG, "unknown repetition rules %d", s->rules);
    if (s->rules == SB_RULES_ISF) {
        if (!s->isf_two_square || !aligned(s->isf_two_square, 8))
            return fail(SB_E_ARG, "SB_RULES_ISF needs an 8-byte aligned isf_two_square [n,600]");
        if (s->two_square_limit < 1 || s->two_square_limit > 3)
            return fail(SB_E_ARG, "SB_RULES_ISF supports two-square limits 1..3");
    }
    if (s->setup_pool && s->pool_size <= 0) return fail(SB_E_ARG, "setup_pool given with pool_size <= 0");
    if (s->pool_size > 0xFFFFFFFFll) return fail(SB_E_ARG, "pool_size above 2^32");
    return SB_OK;
}

sb::KArgs base_args(const sb_state* s) {
    sb::KArgs k;
    memset(&k, 0, sizeof k);
    k.rec = s->records;
    k.ring = s->chase_ring;
    k.zob = s->zobrist;
    k.pool = s->setup_pool;
    k.pool_size = s->pool_size;
    k.n = s->n;
    k.env_base = s->env_base;
    k.seed = s->seed;
    sb::philox_round_keys(s->seed, k.rk);
    k.no_attack_limit = s->no_attack_limit;
    k.max_len = s->max_game_length;
    k.ts_limit = s->two_square_limit;
    k.status = s->status;
    k.rules = s->rules;
    k.isf = s->isf_two_square;
    k.policy = SB_POLICY_UNIFORM;
    k.n_plies = 1;
    k.n_slots = 1;
    k.slot0 = 0;
    return k;
}

struct OccEntry {
    const void* fn;
    int dev;
    int smem;
    int blocks;
};
std::mutex g_mu;
constexpr int CACHE_N = 512;  // kernel instantiations x devices x shared-memory sizes
OccEntry g_occ[CACHE_N];
int g_nocc = 0;
const void* g_attr_fn[CACHE_N];
int g_attr_dev[CACHE_N];
int g_nattr = 0;

// Opt every env_kernel instantiation into the device's full per-block shared
// memory once, then cache the occupancy of each shared-memory size.
int blocks_per_sm(const void* fn, int dev, int smem, int* out) {
    std::lock_guard<std::mutex> lock(g_mu);
    for (int i = 0; i < g_nocc; ++i)
        if (g_occ[i].fn == fn && g_occ[i].dev == dev && g_occ[i].smem == smem) {
            *out = g_occ[i].blocks;
            return SB_OK;
        }
    bool opted = false;
    for (int i = 0; i < g_nattr; ++i)
        if (g_attr_fn[i] == fn && g_attr_dev[i] == dev) opted = true;
    if (!opted) {
        int optin = 0;
        cudaError_t e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
        cudaFuncAttributes fa;
        e = cudaFuncGetAttributes(&fa, fn);
        if (e != cudaSuccess) return cuda_fail(e, "cudaFuncGetAttributes");
        // dynamic shared memory may use what the static part leaves
        e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, optin - (int)fa.sharedSizeBytes);
        if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute");
        if (g_nattr < CACHE_N) {
            g_attr_fn[g_nattr] = fn;
            g_attr_dev[g_nattr++] = dev;
        }
    }
    int nb = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, fn, sb::WARPS * 32, smem);
    if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
    if (nb < 1) return fail(SB_E_CUDA, "kernel does not fit on an SM with %d bytes of shared memory", smem);
    if (g_nocc < CACHE_N) g_occ[g_nocc++] = OccEntry{fn, dev, smem, nb};
    *out = nb;
    return SB_OK;
}

int sm_count(int dev, int* out) {
    static std::atomic<int> cache[64];
    if (dev < 0 || dev >= 64) return fail(SB_E_ARG, "device index out of range");
    int v = cache[dev].load(std::memory_order_relaxed);
    if (!v) {
        cudaError_t e = cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
        cache[dev].store(v, std::memory_order_relaxed);
    }
    *out = v;
    return SB_OK;
}

// Shared memory plan of one warp: record, rays, two hidden-piece rows, and
// the bit buffer of bit-packed masks.
void plan_smem(sb::KArgs& k) {
    int off = sb::SM_FIXED;
    if (k.flags & (sb::F_MASK_BITS | sb::F_MASK_U8)) off += 1264;
    k.sm_warp = (off + 127) / 128 * 128;
}

template <typename T, int MODE>
int launch_mode(sb::KArgs& k, cudaStream_t st) {
    const void* fn = (const void*)sb::env_kernel<T, MODE>;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    const int smem = (MODE == sb::MODE_STEP_PROD ? sb::ZERO_BYTES : 0) + sb::WARPS * k.sm_warp;
    int nb = 0, sms = 0, rc;
    if ((rc = blocks_per_sm(fn, dev, smem, &nb)) != SB_OK) return rc;
    if ((rc = sm_count(dev, &sms)) != SB_OK) return rc;
    const int envw = MODE == sb::MODE_STEP_PROD ? sb::WARPS - 1 : sb::WARPS;
    int64_t blocks = (k.n + envw - 1) / envw;
    const int64_t cap = (int64_t)sms * nb;
    if (blocks > cap) blocks = cap;
    // programmatic dependent launch: this grid's CTAs may become resident
    // while the previous launch on the stream drains; the kernel waits
    // (griddepcontrol.wait) before it touches global memory
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)blocks);
    cfg.blockDim = dim3(sb::WARPS * 32);
    cfg.dynamicSmemBytes = (size_t)smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, sb::env_kernel<T, MODE>, k);
    if (e != cudaSuccess) return cuda_fail(e, "env_kernel launch");
    return SB_OK;
}

// The step kernels (apply + step + propose, one policy) are compiled apart
// from the generic one; everything else goes through MODE_GENERIC.
int launch_env(sb::KArgs& k, int dtype, cudaStream_t st) {
    if (k.n == 0) return SB_OK;
    plan_smem(k);
    const uint32_t step = sb::F_APPLY | sb::F_STEP | sb::F_PROPOSE;
    const uint32_t off = sb::F_RESET_PLANES | sb::F_RESET_POOL | sb::F_SAMPLE_OUT | sb::F_HAS_LEGAL;
    int mode = sb::MODE_GENERIC;
    if ((k.flags & step) == step && !(k.flags & off)) {
        mode = k.policy == SB_POLICY_UNIFORM ? sb::MODE_STEP_UNIFORM : sb::MODE_STEP_GUMBEL;
        if (mode == sb::MODE_STEP_UNIFORM && k.n_plies == 1 && (k.flags & (sb::F_INFO | sb::F_MASK_U8)) &&
            k.rules == SB_RULES_CUDA)
            mode = sb::MODE_STEP_PROD;
        if (k.rules == SB_RULES_ISF) mode |= sb::MODE_ISF;
    }
    const bool f32 = dtype == SB_DTYPE_F32;
    constexpr int UI = sb::MODE_STEP_UNIFORM | sb::MODE_ISF, GI = sb::MODE_STEP_GUMBEL | sb::MODE_ISF;
    switch (mode) {
        case sb::MODE_STEP_UNIFORM:
            return f32 ? launch_mode<float, sb::MODE_STEP_UNIFORM>(k, st) : launch_mode<uint16_t, sb::MODE_STEP_UNIFORM>(k, st);
        case sb::MODE_STEP_GUMBEL:
            return f32 ? launch_mode<float, sb::MODE_STEP_GUMBEL>(k, st) : launch_mode<uint16_t, sb::MODE_STEP_GUMBEL>(k, st);
        case UI:
            return f32 ? launch_mode<float, UI>(k, st) : launch_mode<uint16_t, UI>(k, st);
        case GI:
            return f32 ? launch_mode<float, GI>(k, st) : launch_mode<uint16_t, GI>(k, st);
        case sb::MODE_STEP_PROD:
            return f32 ? launch_mode<float, sb::MODE_STEP_PROD>(k, st) : launch_mode<uint16_t, sb::MODE_STEP_PROD>(k, st);
        default:
            return f32 ? launch_mode<float, sb::MODE_GENERIC>(k, st) : launch_mode<uint16_t, sb::MODE_GENERIC>(k, st);
    }
}

int check_info(const void* p, int dtype, int layout) {
    if (dtype != SB_DTYPE_F32 && dtype != SB_DTYPE_BF16) return fail(SB_E_ARG, "bad infostate dtype %d", dtype);
    if (layout < SB_LAYOUT_DENSE_ALL || layout > SB_LAYOUT_COMPACT) return fail(SB_E_ARG, "bad infostate layout %d", layout);
    if (!aligned(p, 16)) return fail(SB_E_ARG, "infostate buffer not 16-byte aligned");
    return SB_OK;
}

int check_policy(const sb_policy* pol) {
    if (!pol) return SB_OK;
    if (pol->kind != SB_POLICY_UNIFORM && pol->kind != SB_POLICY_GUMBEL) return fail(SB_E_ARG, "bad policy %d", pol->kind);
    if (pol->logits && pol->kind != SB_POLICY_GUMBEL) return fail(SB_E_ARG, "logits need SB_POLICY_GUMBEL");
    return SB_OK;
}

// Device address of g_noalloc_actions on the current device, looked up on
// the first call per device.
std::mutex g_noalloc_mu;
int64_t* g_noalloc_addr[64];
int noalloc_staging(int64_t** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    if (dev < 0 || dev >= 64) return fail(SB_E_ARG, "device index out of range");
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_addr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_actions);
        if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress of the staging array");
        g_noalloc_addr[dev] = static_cast<int64_t*>(p);
    }
    *out = g_noalloc_addr[dev];
    return SB_OK;
}

}  // namespace

extern "C" {

int sb_abi_version(void) { return SB_ABI_VERSION; }

int sb_debug_bounds(void) { return sb::kDebugBounds ? 1 : 0; }

const char* sb_last_error(void) { return g_err; }

int sb_hello_world(int32_t* out, void* stream) {
    if (!out) return fail(SB_E_ARG, "out is NULL");
    sb::hello_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(out);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? SB_OK : cuda_fail(e, "hello_kernel launch");
}

int sb_init_state(const sb_state* s, void* stream) {
    int rc = check_state(s);
    if (rc != SB_OK || s->n == 0) return rc;
    const int64_t blocks = (s->n + 127) / 128;
    sb::init_kernel<<<(unsigned)blocks, 128, 0, (cudaStream_t)stream>>>(s->records, s->chase_ring, s->n, s->rules,
                                                                        s->isf_two_square);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? SB_OK : cuda_fail(e, "init_kernel launch");
}

int sb_reset_planes(const sb_state* s, const int8_t* setup_red, const int8_t* setup_blue, int force_all,
                    void* stream) {
    int rc = check_state(s);
    if (rc != SB_OK || s->n == 0) return rc;
    if (!setup_red || !setup_blue) return fail(SB_E_ARG, "setup planes are NULL");
    sb::KArgs k = base_args(s);
    k.flags = sb::F_RESET_PLANES | (force_all ? sb::F_FORCE : 0);
    k.setup_red = setup_red;
    k.setup_blue = setup_blue;
    return launch_env(k, SB_DTYPE_F32, (cudaStream_t)stream);
}

int sb_reset_pool(const sb_state* s, int force_all, void* stream) {
    int rc = check_state(s);
    if (rc != SB_OK || s->n == 0) return rc;
    if (!s->setup_pool) return fail(SB_E_NOPOOL, "no setup pool");
    sb::KArgs k = base_args(s);
    k.flags = sb::F_RESET_POOL | (force_all ? sb::F_FORCE : 0);
    return launch_env(k, SB_DTYPE_F32, (cudaStream_t)stream);
}

int sb_make_setup_pool(uint64_t seed, int64_t start, int64_t count, uint8_t* out, void* stream) {
    if (count < 0 || start < 0) return fail(SB_E_ARG, "negative pool range");
    if (count == 0) return SB_OK;
    if (!out) return fail(SB_E_ARG, "out is NULL");
    const int64_t blocks = (count + 127) / 128;
    sb::pool_kernel<<<(unsigned)blocks, 128, 0, (cudaStream_t)stream>>>(seed, start, count, out);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? SB_OK : cuda_fail(e, "pool_kernel launch");
}

int sb_apply_actions(const sb_state* s, const int64_t* actions, void* stream) {
    int rc = check_state(s);
    if (rc != SB_OK || s->n == 0) return rc;
    if (!actions) return fail(SB_E_ARG, "actions is NULL");
    sb::KArgs k = base_args(s);
    k.flags = sb::F_APPLY;
    k.actions = actions;
    return launch_env(k, SB_DTYPE_F32, (cudaStream_t)stream);
}

int sb_step(const sb_state* s, const int64_t* actions, int64_t ply, const sb_policy* policy, int auto_reset,
            const sb_step_out* out, void* stream) {
    int rc = check_state(s);
    if (rc != SB_OK || s->n == 0) return rc;
    if ((rc = check_policy(policy)) != SB_OK) return rc;
    if (auto_reset && !s->setup_pool) return fail(SB_E_NOPOOL, "auto_reset needs a setup pool");
    sb_step_out o;
    memset(&o, 0, sizeof o);
    if (out) o = *out;
    sb::KArgs k = base_args(s);
    k.flags = sb::F_APPLY | sb::F_STEP | sb::F_PROPOSE | (auto_reset ? sb::F_AUTO_RESET : 0);
    k.actions = actions;
    k.ply = ply;
    k.propose_ply = ply + 1;
    if (policy) {
        k.policy = policy->kind;
        k.logits = policy->logits;
    }
    int dtype = SB_DTYPE_F32;
    if (o.infostate) {
        if ((rc = check_info(o.infostate, o.info_dtype, o.info_layout)) != SB_OK) return rc;
        k.flags |= sb::F_INFO;
        k.info = o.infostate;
        k.info_layout = o.info_layout;
        dtype = o.info_dtype;
    }
    if (o.mask_u8) {
        if (!aligned(o.mask_u8, 16)) return fail(SB_E_ARG, "mask_u8 not 16-byte aligned");
        k.flags |= sb::F_MASK_U8;
        k.mask_u8 = o.mask_u8;
    }
    if (o.mask_bits) {
        if (!aligned(o.mask_bits, 2)) return fail(SB_E_ARG, "mask_bits not 2-byte aligned");
        k.flags |= sb::F_MASK_BITS;
        k.mask_bits = o.mask_bits;
    }
    if (o.hash) k.flags |= sb::F_HASH;
    k.hash = o.hash;
    k.reward = o.reward;
    k.done = o.done;
    k.action_taken = o.action_taken;
    k.logprob_taken = o.logprob_taken;
    k.next_action = o.next_action;
    k.next_logprob = o.next_logprob;
    k.stats = o.stats;
    return launch_env(k, dtype, (cudaStream_t)stream);
}

// Address through which a kernel reaches p: device and managed memory as
// is, page-locked host memory through its device mapping; SB_E_ARG for
// pageable host memory (a kernel touching it would fault).
static int device_view(const void* p, void** dev) {
    cudaPointerAttributes at;
    cudaError_t e = cudaPointerGetAttributes(&at, p);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(SB_E_ARG, "pointer is neither device memory nor page-locked host memory");
    }
    if (at.type == cudaMemoryTypeDevice || at.type == cudaMemoryTypeManaged) {
        *dev = const_cast<void*>(p);
        return SB_OK;
    }
    if (at.type != cudaMemoryTypeHost || !at.devicePointer)
        return fail(SB_E_ARG, "pointer is neither device memory nor page-locked host memory");
    *dev = at.devicePointer;
    return SB_OK;
}

int sb_step_host(const sb_state* s, const sb_host_io* io, int64_t ply, const sb_policy* policy, int auto_reset,
                 const sb_step_out* out, void* stream) {
    int rc = check_state(s);
    if (rc != SB_OK) return rc;
    if (!io) return fail(SB_E_ARG, "io is NULL");
    if (io->back_bytes < 0 || (io->back_bytes > 0 && (!io->back_dev || !io->back_host)))
        return fail(SB_E_ARG, "bad copy-back range");
    cudaStream_t st = (cudaStream_t)stream;
    const int64_t* acts = nullptr;
    if (io->actions_host && io->actions_dev) {
        if (s->n > 0) {
            cudaError_t e = cudaMemcpyAsync(io->actions_dev, io->actions_host, (size_t)s->n * sizeof(int64_t),
                                            cudaMemcpyHostToDevice, st);
            if (e != cudaSuccess) return cuda_fail(e, "actions host->device");
        }
        acts = io->actions_dev;
    } else if (io->actions_host) {
        // read in place by the kernel
        void* d = nullptr;
        if ((rc = device_view(io->actions_host, &d)) != SB_OK) return rc;
        acts = static_cast<const int64_t*>(d);
    }
    sb_step_out o;
    memset(&o, 0, sizeof o);
    if (out) o = *out;
    if (io->back_bytes == 0) {
        // no copy back: the per-env results may live in page-locked host memory
        void* d = nullptr;
        if (o.reward && (rc = device_view(o.reward, &d)) == SB_OK) o.reward = static_cast<float*>(d);
        if (rc == SB_OK && o.done && (rc = device_view(o.done, &d)) == SB_OK) o.done = static_cast<uint8_t*>(d);
        if (rc == SB_OK && o.next_action && (rc = device_view(o.next_action, &d)) == SB_OK)
            o.next_action = static_cast<int16_t*>(d);
        if (rc != SB_OK) return rc;
    }
    rc = sb_step(s, acts, ply, policy, auto_reset, &o, stream);
    if (rc != SB_OK) return rc;
    if (io->back_bytes > 0) {
        cudaError_t e = cudaMemcpyAsync(io->back_host, io->back_dev, (size_t)io->back_bytes,
                                        cudaMemcpyDeviceToHost, st);
        if (e != cudaSuccess) return cuda_fail(e, "results device->host");
    }
    if (io->sync) {
        cudaError_t e = cudaStreamSynchronize(st);
        if (e != cudaSuccess) return cuda_fail(e, "stream synchronize");
    }
    return SB_OK;
}

int sb_step_host_noalloc(const sb_state* s, const sb_host_io* io, int64_t ply, const sb_policy* policy,
                         int auto_reset, const sb_step_out* out, void* stream) {
    int rc = check_state(s);
    if (rc != SB_OK) return rc;
    if (!io) return fail(SB_E_ARG, "io is NULL");
    if (io->actions_dev) return fail(SB_E_ARG, "actions_dev must be NULL: the library stages the actions itself");
    if (s->n > SB_NOALLOC_MAX_ENVS)
        return fail(SB_E_ARG, "%lld envs: at most %d per call without allocation", (long long)s->n, SB_NOALLOC_MAX_ENVS);
    if (s->n > 0 && io->actions_host) {
        // the staging array used is the current device's: the games must live there
        int dev = 0;
        cudaPointerAttributes at;
        cudaError_t e = cudaGetDevice(&dev);
        if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
        e = cudaPointerGetAttributes(&at, s->records);
        if (e != cudaSuccess) {
            cudaGetLastError();
            return fail(SB_E_ARG, "records are not device memory");
        }
        if (at.type != cudaMemoryTypeDevice || at.device != dev)
            return fail(SB_E_ARG, "records live on device %d, but device %d is current", at.device, dev);
    }
    sb_host_io local = *io;
    if (io->actions_host && (rc = noalloc_staging(&local.actions_dev)) != SB_OK) return rc;
    return sb_step_host(s, &local, ply, policy, auto_reset, out, stream);
}

int sb_serve_start(const sb_state* s, int64_t ply0, int auto_reset, const int64_t* actions_host,
                   const sb_step_out* out, sb_serve* sv, void* stream) {
    int rc = check_state(s);
    if (rc != SB_OK) return rc;
    if (!sv || !sv->ctl || !sv->dev || !out) return fail(SB_E_ARG, "serve control blocks or outputs are NULL");
    if (!aligned(sv->dev, 8)) return fail(SB_E_ARG, "serve device relay not 8-byte aligned");
    if (s->n < 1) return fail(SB_E_ARG, "no envs");
    if (s->rules != SB_RULES_CUDA) return fail(SB_E_ARG, "the step server runs the CUDA repetition rules");
    if (sv->limit_ns <= 0) return fail(SB_E_ARG, "limit_ns must be > 0");
    if (auto_reset && !s->setup_pool) return fail(SB_E_NOPOOL, "auto_reset needs a setup pool");
    sb_step_out o = *out;
    if (!o.infostate && !o.mask_u8) return fail(SB_E_ARG, "the step server writes an infostate and / or a u8 mask");
    if (o.mask_bits || o.hash) return fail(SB_E_ARG, "the step server writes no bit-packed mask or hash");
    void* d = nullptr;
    if ((rc = device_view(sv->ctl, &d)) != SB_OK) return rc;
    int64_t* ctl = static_cast<int64_t*>(d);
    const int64_t* acts = nullptr;
    if (actions_host) {
        if ((rc = device_view(actions_host, &d)) != SB_OK) return rc;
        acts = static_cast<const int64_t*>(d);
    }
    if (sv->back_bytes < 0 || sv->back_bytes % 16 || (sv->back_bytes && (!sv->back_dev || !sv->back_host)) ||
        !aligned(sv->back_dev, 16) || !aligned(sv->back_host, 16))
        return fail(SB_E_ARG, "bad copy-back range (16-byte aligned, a multiple of 16 bytes)");
    void* back_host = nullptr;
    if (sv->back_bytes && (rc = device_view(sv->back_host, &back_host)) != SB_OK) return rc;
    if (o.infostate && (rc = check_info(o.infostate, o.info_dtype, o.info_layout)) != SB_OK) return rc;
    if (o.mask_u8 && !aligned(o.mask_u8, 16)) return fail(SB_E_ARG, "mask_u8 not 16-byte aligned");
    sb::KArgs k = base_args(s);
    k.flags = sb::F_APPLY | sb::F_STEP | sb::F_PROPOSE | (auto_reset ? sb::F_AUTO_RESET : 0);
    k.actions = acts;
    k.ply = ply0;
    k.propose_ply = ply0 + 1;
    k.policy = SB_POLICY_UNIFORM;
    int dtype = SB_DTYPE_F32;
    if (o.infostate) {
        k.flags |= sb::F_INFO;
        k.info = o.infostate;
        k.info_layout = o.info_layout;
        dtype = o.info_dtype;
    }
    if (o.mask_u8) {
        k.flags |= sb::F_MASK_U8;
        k.mask_u8 = o.mask_u8;
    }
    k.action_taken = o.action_taken;
    k.logprob_taken = o.logprob_taken;
    k.next_logprob = o.next_logprob;
    k.stats = o.stats;
    k.serve_ctl = ctl;
    k.serve_dev = sv->dev;
    k.reward = o.reward;
    k.done = o.done;
    k.next_action = o.next_action;
    k.serve_back_dev = static_cast<const uint8_t*>(sv->back_dev);
    k.serve_back_host = static_cast<uint8_t*>(back_host);
    k.serve_back_bytes = sv->back_bytes;
    k.serve_limit_ns = sv->limit_ns;
    plan_smem(k);
    constexpr int SV = sb::MODE_STEP_PROD | sb::MODE_SERVE;
    const void* fn = dtype == SB_DTYPE_F32 ? (const void*)sb::env_kernel<float, SV> : (const void*)sb::env_kernel<uint16_t, SV>;
    int dev = 0, nb = 0, sms = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    const int smem = sb::ZERO_BYTES + sb::WARPS * k.sm_warp;
    if ((rc = blocks_per_sm(fn, dev, smem, &nb)) != SB_OK) return rc;
    if ((rc = sm_count(dev, &sms)) != SB_OK) return rc;
    const int64_t blocks = (s->n + sb::WARPS - 2) / (sb::WARPS - 1);
    if (blocks > (int64_t)sms * nb)
        return fail(SB_E_ARG, "%lld envs need %lld resident CTAs; this GPU holds %lld", (long long)s->n,
                    (long long)blocks, (long long)sms * nb);
    memset(sv->ctl, 0, 17 * sizeof(int64_t));
    e = cudaMemsetAsync(sv->dev, 0, 4 * sizeof(int64_t), (cudaStream_t)stream);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync");
    sv->n_ctas = blocks;
    void* args[] = {&k};
    // cooperative: every CTA resident at once (the host waits for all of them)
    e = cudaLaunchCooperativeKernel(fn, dim3((unsigned)blocks), dim3(sb::WARPS * 32), args, (size_t)smem,
                                    (cudaStream_t)stream);
    return e == cudaSuccess ? SB_OK : cuda_fail(e, "step server launch");
}

int sb_serve_step(const sb_serve* sv, int64_t t, int64_t timeout_ns) {
    if (!sv || !sv->ctl || sv->n_ctas < 1) return fail(SB_E_ARG, "no running step server");
    __atomic_store_n(sv->ctl + sb::SERVE_GO, t, __ATOMIC_RELEASE);
    timespec t0, now;
    clock_gettime(CLOCK_MONOTONIC, &t0);
    while (__atomic_load_n(sv->ctl + sb::SERVE_DONE, __ATOMIC_ACQUIRE) < t) {
        clock_gettime(CLOCK_MONOTONIC, &now);
        const int64_t dt = (int64_t)(now.tv_sec - t0.tv_sec) * 1000000000ll + (now.tv_nsec - t0.tv_nsec);
        if (dt > timeout_ns) return fail(SB_E_CUDA, "step %lld not finished in time", (long long)t);
    }
    return SB_OK;
}

int sb_serve_stop(const sb_serve* sv, int64_t t_done, void* stream) {
    if (!sv || !sv->ctl) return fail(SB_E_ARG, "no step server");
    __atomic_store_n(sv->ctl + sb::SERVE_STOP, (int64_t)1, __ATOMIC_RELEASE);
    __atomic_store_n(sv->ctl + sb::SERVE_GO, t_done + 1, __ATOMIC_RELEASE);
    cudaError_t e = cudaStreamSynchronize((cudaStream_t)stream);
    return e == cudaSuccess ? SB_OK : cuda_fail(e, "step server stop");
}

int sb_rollout(const sb_state* s, int64_t ply, const sb_policy* policy, int auto_reset, int32_t n_plies,
               const sb_traj* traj, void* stream) {
    int rc = check_state(s);
    if (rc != SB_OK || s->n == 0) return rc;
    if ((rc = check_policy(policy)) != SB_OK) return rc;
    if (!traj) return fail(SB_E_ARG, "traj is NULL");
    if (n_plies < 0) return fail(SB_E_ARG, "n_plies < 0");
    if (traj->n_slots < 1 || traj->n_slots > 0x7FFFFFFFll || traj->slot0 < 0)
        return fail(SB_E_ARG, "bad trajectory ring (n_slots outside 1..2^31-1, or slot0 < 0)");
    if (policy && policy->logits && n_plies > 1) return fail(SB_E_ARG, "logits in memory cover one ply only");
    if (auto_reset && n_plies > 0 && !s->setup_pool) return fail(SB_E_NOPOOL, "auto_reset needs a setup pool");
    sb::KArgs k = base_args(s);
    k.flags = sb::F_APPLY | sb::F_STEP | sb::F_PROPOSE | (auto_reset ? sb::F_AUTO_RESET : 0);
    k.ply = ply;
    k.n_plies = n_plies;
    k.n_slots = (int32_t)traj->n_slots;
    k.slot0 = (int32_t)(traj->slot0 % traj->n_slots);
    if (policy) {
        k.policy = policy->kind;
        k.logits = policy->logits;
    }
    int dtype = SB_DTYPE_F32;
    if (traj->infostate) {
        if ((rc = check_info(traj->infostate, traj->info_dtype, traj->info_layout)) != SB_OK) return rc;
        k.flags |= sb::F_INFO;
        k.info = traj->infostate;
        k.info_layout = traj->info_layout;
        dtype = traj->info_dtype;
    }
    if (traj->mask_u8) {
        if (!aligned(traj->mask_u8, 16)) return fail(SB_E_ARG, "mask_u8 not 16-byte aligned");
        k.flags |= sb::F_MASK_U8;
        k.mask_u8 = traj->mask_u8;
    }
    if (traj->mask_bits) {
        if (!aligned(traj->mask_bits, 2)) return fail(SB_E_ARG, "mask_bits not 2-byte aligned");
        k.flags |= sb::F_MASK_BITS;
        k.mask_bits = traj->mask_bits;
    }
    if (traj->hash) k.flags |= sb::F_HASH;
    k.hash = traj->hash;
    k.next_action = traj->action;
    k.next_logprob = traj->logprob;
    k.reward = traj->reward;
    k.done = traj->done;
    k.stats = traj->stats;
    return launch_env(k, dtype, (cudaStream_t)stream);
}

int sb_belief_resample(const sb_state* roots, const sb_state* samples, const int64_t* root_of, void* stream) {
    int rc = check_state(roots);
    if (rc != SB_OK) return rc;
    if ((rc = check_state(samples)) != SB_OK) return rc;
    if (samples->n == 0) return SB_OK;
    if (roots->n < 1) return fail(SB_E_ARG, "no roots");
    if (!root_of) return fail(SB_E_ARG, "root_of is NULL");
    if (roots->rules != samples->rules) return fail(SB_E_ARG, "roots and samples follow different repetition rules");
    sb::KArgs k = base_args(samples);
    int dev = 0, sms = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    if ((rc = sm_count(dev, &sms)) != SB_OK) return rc;
    int64_t blocks = (samples->n + sb::WARPS - 1) / sb::WARPS;
    if (blocks > (int64_t)sms * 16) blocks = (int64_t)sms * 16;
    sb::belief_kernel<<<(unsigned)blocks, sb::WARPS * 32, 0, (cudaStream_t)stream>>>(roots->records, roots->n, root_of, k,
                                                                                   roots->isf_two_square);
    e = cudaGetLastError();
    return e == cudaSuccess ? SB_OK : cuda_fail(e, "belief_kernel launch");
}

int sb_sample_actions(const sb_state* s, int64_t ply, const sb_policy* policy, int64_t* actions, float* logprob,
                      void* stream) {
    int rc = check_state(s);
    if (rc != SB_OK || s->n == 0) return rc;
    if ((rc = check_policy(policy)) != SB_OK) return rc;
    sb::KArgs k = base_args(s);
    k.flags = sb::F_SAMPLE_OUT;
    k.ply = ply;
    if (policy) {
        k.policy = policy->kind;
        k.logits = policy->logits;
    }
    k.sampled = actions;
    k.sampled_lp = logprob;
    return launch_env(k, SB_DTYPE_F32, (cudaStream_t)stream);
}

int sb_legal_mask_u8(const sb_state* s, uint8_t* mask, void* stream) {
    int rc = check_state(s);
    if (rc != SB_OK || s->n == 0) return rc;
    if (!mask || !aligned(mask, 16)) return fail(SB_E_ARG, "mask NULL or not 16-byte aligned");
    sb::KArgs k = base_args(s);
    k.flags = sb::F_MASK_U8;
    k.mask_u8 = mask;
    return launch_env(k, SB_DTYPE_F32, (cudaStream_t)stream);
}

int sb_legal_mask_bits(const sb_state* s, uint8_t* bits, void* stream) {
    int rc = check_state(s);
    if (rc != SB_OK || s->n == 0) return rc;
    if (!bits || !aligned(bits, 2)) return fail(SB_E_ARG, "bits NULL or not 2-byte aligned");
    sb::KArgs k = base_args(s);
    k.flags = sb::F_MASK_BITS;
    k.mask_bits = bits;
    return launch_env(k, SB_DTYPE_F32, (cudaStream_t)stream);
}

int sb_infostate(const sb_state* s, void* out, int dtype, int layout, void* stream) {
    int rc = check_state(s);
    if (rc != SB_OK || s->n == 0) return rc;
    if (!out) return fail(SB_E_ARG, "out is NULL");
    if ((rc = check_info(out, dtype, layout)) != SB_OK) return rc;
    sb::KArgs k = base_args(s);
    k.flags = sb::F_INFO;
    k.info = out;
    k.info_layout = layout;
    return launch_env(k, dtype, (cudaStream_t)stream);
}

int sb_hash_board(const sb_state* s, int64_t* out, void* stream) {
    int rc = check_state(s);
    if (rc != SB_OK || s->n == 0) return rc;
    if (!out) return fail(SB_E_ARG, "out is NULL");
    sb::KArgs k = base_args(s);
    k.flags = sb::F_HASH;
    k.hash = out;
    return launch_env(k, SB_DTYPE_F32, (cudaStream_t)stream);
}

int sb_has_legal_movement(const sb_state* s, uint8_t* out, void* stream) {
    int rc = check_state(s);
    if (rc != SB_OK || s->n == 0) return rc;
    if (!out) return fail(SB_E_ARG, "out is NULL");
    sb::KArgs k = base_args(s);
    k.flags = sb::F_HAS_LEGAL;
    k.has_legal = out;
    return launch_env(k, SB_DTYPE_F32, (cudaStream_t)stream);
}

int sb_export_state(const sb_state* s, const sb_export* out, void* stream) {
    int rc = check_state(s);
    if (rc != SB_OK || s->n == 0) return rc;
    if (!out) return fail(SB_E_ARG, "out is NULL");
    const int64_t blocks = (s->n + 127) / 128;
    sb::export_kernel<<<(unsigned)blocks, 128, 0, (cudaStream_t)stream>>>(s->records, s->n, *out, s->rules,
                                                                          s->isf_two_square);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? SB_OK : cuda_fail(e, "export_kernel launch");
}

int sb_sum_move_number(const sb_state* s, int64_t* out, void* stream) {
    int rc = check_state(s);
    if (rc != SB_OK) return rc;
    if (!out) return fail(SB_E_ARG, "out is NULL");
    cudaError_t e = cudaMemsetAsync(out, 0, sizeof(int64_t), (cudaStream_t)stream);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync");
    if (s->n == 0) return SB_OK;
    int64_t blocks = (s->n + 255) / 256;
    if (blocks > 1024) blocks = 1024;
    sb::sum_move_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(s->records, s->n, out);
    e = cudaGetLastError();
    return e == cudaSuccess ? SB_OK : cuda_fail(e, "sum_move_kernel launch");
}

}  // extern "C"
