/*
 * stratego_b200.h -- C ABI of the B200 StrategoRolloutBuffer simulator.
 *
 * One shared library, libstratego_b200.so, built for sm_100a.  Every entry
 * point takes plain device pointers, sizes and a cudaStream_t (passed as
 * void*), launches on that stream and returns 0 on success or a negative
 * SB_E_* code (sb_last_error() gives the message).  Nothing here allocates
 * device memory: the caller owns every buffer (the Python host class in
 * ataraxos_b200/buffer.py allocates them with torch).
 *
 * Each entry point replaces one piece of the reference's pybind class
 * _stratego_cuda.StrategoRolloutBuffer (csrc/stratego_buffer.cpp) or one of
 * its launchers (csrc/stratego_buffer.cuh); the reference line is cited on
 * each declaration.  Entry points marked "north-star" have no reference
 * counterpart: they are the step / setup-pool / sampling / trajectory
 * contract the build adds around the same state.
 *
 * Game state lives in one record of SB_RECORD_BYTES bytes per env (board,
 * counters, trackers, move-history ring) plus the per-side 64-entry chase
 * ring (int64 [n,2,64]); sb_export_state() writes it out in the reference's
 * own tensor layout (csrc/stratego_buffer.cpp:24-55).
 */
#ifndef STRATEGO_B200_H
#define STRATEGO_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SB_ABI_VERSION 2
#define SB_RECORD_BYTES 256
#define SB_NUM_SQUARES 100
#define SB_NUM_ACTIONS 10000
#define SB_NUM_CHANNELS 488
#define SB_LIVE_CHANNELS 75      /* channels 0-42 and 456-487 */
#define SB_COMPACT_CHANNELS 76   /* 0-42, one zero pad plane, 456-487 */
#define SB_MASK_BITS_BYTES 1250  /* bit j of byte k = flat action 8k+j */
#define SB_SETUP_BYTES 40        /* one pool entry: piece type per home slot */

/* error codes */
#define SB_OK 0
#define SB_E_ARG (-1)      /* bad argument (null pointer, size, alignment) */
#define SB_E_CUDA (-2)     /* a CUDA runtime call failed */
#define SB_E_NOPOOL (-3)   /* a pool reset was asked for without a pool */

/* infostate element type and layout */
#define SB_DTYPE_F32 0
#define SB_DTYPE_BF16 1
#define SB_LAYOUT_DENSE_ALL 0  /* [n,488,10,10]; every channel written */
#define SB_LAYOUT_DENSE_LIVE 1 /* [n,488,10,10]; only channels 0-42, 456-487 written
                                  (43-455 must already be zero) */
#define SB_LAYOUT_COMPACT 2    /* [n,76,10,10]; plane 43 is a zero pad that the
                                  caller zeroes once */

/* repetition rules (sb_state.rules) */
#define SB_RULES_CUDA 0        /* the reference CUDA class's trackers: two-square per mover,
                                  chasing on every threatening move (csrc/stratego_buffer.cu:272-381) */
#define SB_RULES_ISF 1         /* the reference Python trackers (ISF rules): two-square per piece with
                                  scout pairs (stratego/env/two_square.py:27-94), chasing gated on the
                                  opponent's evasions (stratego/env/chasing.py:54-109); needs
                                  isf_two_square and a two-square limit of 1..3 */

/* action policies for sampling */
#define SB_POLICY_UNIFORM 0    /* k = (u32 * n_legal) >> 32 over ascending legal actions */
#define SB_POLICY_GUMBEL 1     /* argmax(logit + Gumbel) over legal actions; logits are
                                  read from memory when given, else virtual N(0,1) */

/* Device-side state of a shard of envs.  Plain pointers and sizes only. */
typedef struct sb_state {
    uint8_t *records;          /* [n, SB_RECORD_BYTES], 16-byte aligned */
    int64_t *chase_ring;       /* [n, 2, 64] */
    const int64_t *zobrist;    /* [10,10,2,13] Zobrist table */
    const uint8_t *setup_pool; /* [pool_size, 40] or NULL */
    int64_t pool_size;
    int64_t n;                 /* envs in this shard */
    int64_t env_base;          /* global index of env 0 (keys the RNG streams) */
    uint64_t seed;             /* Philox key */
    int32_t no_attack_limit;   /* draw after this many plies without combat (100) */
    int32_t max_game_length;   /* draw at this ply count (4000) */
    int32_t two_square_limit;  /* violation above this many repeats (3) */
    int32_t rules;             /* SB_RULES_* */
    int32_t *status;           /* device word; kernels OR SB_STATUS_* bits in (may be NULL) */
    uint8_t *isf_two_square;   /* [n,100,6] per-square two-square state of SB_RULES_ISF
                                  (NULL under SB_RULES_CUDA) */
} sb_state;

#define SB_STATUS_BAD_SETUP 1   /* a setup plane or pool entry held a piece code > 12 */
#define SB_STATUS_WAIT_TIMEOUT 2 /* a kernel gave up waiting (about 1 s) on an in-CTA handshake */
#define SB_STATUS_BAD_STATE 4   /* debug build only: a game record failed its bounds checks (a piece
                                   code, a history / chase-ring head, length or entry, a square or
                                   action index out of range); that game was skipped, untouched */

/* Outputs of one fused step; any pointer may be NULL (not produced). */
typedef struct sb_step_out {
    uint8_t *mask_u8;          /* [n,100,100] legal mask of the new state */
    uint8_t *mask_bits;        /* [n,1250] bit-packed legal mask of the new state */
    void *infostate;           /* infostate of the new state, see info_dtype/info_layout */
    int32_t info_dtype;
    int32_t info_layout;
    float *reward;             /* [n] reward for player 0 of this transition */
    uint8_t *done;             /* [n] 1 if the transition ended the game */
    int64_t *action_taken;     /* [n] action applied this step (-1 none) */
    float *logprob_taken;      /* [n] log-prob of the applied action when sampled */
    int16_t *next_action;      /* [n] action proposed for the new state (-1 none: no legal
                                  move, or the game is over and was not reset) */
    float *next_logprob;       /* [n] its log-prob */
    int64_t *hash;             /* [n] Zobrist hash of the new board */
    int64_t *stats;            /* [5] accumulated over games that ended this step:
                                  finished, red wins, blue wins, draws, sum of lengths */
} sb_step_out;

/* Policy / action source of a step. */
typedef struct sb_policy {
    int32_t kind;              /* SB_POLICY_* */
    int32_t reserved;
    const float *logits;       /* [n,10000] or NULL (virtual Philox N(0,1)) */
} sb_policy;

/* ---- version / errors ------------------------------------------------ */
int sb_abi_version(void);
const char *sb_last_error(void);
/* 1 in the debug build (libstratego_b200_debug.so, compiled with
 * -DSB_DEBUG_BOUNDS): every kernel that plays or observes a game first checks
 * its record's indices and skips a bad game with SB_STATUS_BAD_STATE instead
 * of reading or writing out of range.  0 in the production build, which
 * trusts records that only its own kernels (or sb_init_state / resets) wrote. */
int sb_debug_bounds(void);

/* ---- construction ------------------------------------------------------
 * Initial state of a fresh buffer: empty board, Red to move, outcome ongoing,
 * trackers at their reset values (csrc/stratego_buffer.cpp:24-55). */
int sb_init_state(const sb_state *s, void *stream);

/* hello_world kernel: writes 42 to out[0] (csrc/stratego_buffer.cu:65-76,
 * csrc/stratego_buffer.cpp:59-67). */
int sb_hello_world(int32_t *out, void *stream);

/* ---- resets ------------------------------------------------------------
 * reset_terminated / reset_all from setup planes (csrc/stratego_buffer.cu:529-618,
 * csrc/stratego_buffer.cpp:245-298): for terminated envs (every env when
 * force_all != 0) rebuild the board from setup_red/setup_blue [n,10,10] int8
 * (non-zero = piece, red first), Red to move, trackers cleared, and
 * flag_captured / terminated_since cleared. */
int sb_reset_planes(const sb_state *s, const int8_t *setup_red, const int8_t *setup_blue, int force_all,
                    void *stream);

/* north-star: same reset, with each env's setups drawn from the device setup
 * pool by Philox(seed; global env index, episode). */
int sb_reset_pool(const sb_state *s, int force_all, void *stream);

/* north-star: fill pool entries [start, start+count) for `seed`
 * (Fisher-Yates over the 40-piece roster driven by Philox4x32-10). */
int sb_make_setup_pool(uint64_t seed, int64_t start, int64_t count, uint8_t *out, void *stream);

/* ---- one ply ------------------------------------------------------------
 * apply_actions (csrc/stratego_buffer.cu:82-400, csrc/stratego_buffer.cpp:70-120):
 * validate and apply actions[n] (src*100+dst, int64); illegal actions are
 * ignored for that env (its invalid counter counts them); flag_captured and
 * terminated_since updated as the reference's host wrapper does. */
int sb_apply_actions(const sb_state *s, const int64_t *actions, void *stream);

/* north-star: the fused ply.  actions == NULL samples each env's action at
 * `ply` with `policy`; then apply, per-env auto-reset from the pool when
 * auto_reset != 0, then every requested output of the new state, all in one
 * kernel.  The proposal for the next ply is cached in the record. */
int sb_step(const sb_state *s, const int64_t *actions, int64_t ply, const sb_policy *policy, int auto_reset,
            const sb_step_out *out, void *stream);

/* Host side of one ply, for callers whose actions and results live in host
 * memory (the reference's apply_actions takes host tensors and copies them
 * in, csrc/stratego_buffer.cpp:70-80; its getters copy back, cpp:300-338). */
typedef struct sb_host_io {
    const int64_t *actions_host; /* pinned host int64[n], or NULL to sample on the device */
    int64_t *actions_dev;        /* device int64[n] the host actions are copied into; NULL: the
                                    kernel reads actions_host in place (it must be page-locked
                                    memory mapped for the device, else SB_E_ARG) */
    const void *back_dev;        /* device range copied to back_host after the step; lay the */
    void *back_host;             /*   step_out fields the host reads (reward, done, next_action) */
    int64_t back_bytes;          /*   out contiguously so that one copy brings them back (0: no
                                    copy, e.g. when those step_out fields point at mapped
                                    page-locked host memory that the kernel writes directly) */
    int32_t sync;                /* nonzero: return once the step (and copy back) has landed */
    int32_t reserved;
} sb_host_io;

/* north-star: sb_step with the host transfers folded into the same call:
 * actions_host -> actions_dev (or read in place), the fused ply,
 * back_dev -> back_host, all in stream order on `stream` (no allocation). */
int sb_step_host(const sb_state *s, const sb_host_io *io, int64_t ply, const sb_policy *policy, int auto_reset,
                 const sb_step_out *out, void *stream);

/* No counterpart in the reference.  sb_step_host for callers that cannot
 * allocate device memory for the staging copy of their host actions: code
 * running inside another framework's fixed memory plan, which hands this
 * library only the state and output buffers it planned, or a latency-bound
 * loop that must not call cudaMalloc (it can synchronise the device).  The
 * host actions are copied into a staging array built into the library (a
 * file-scope device array of SB_NOALLOC_MAX_ENVS int64 entries, 2 MiB, held
 * by every GPU that loads the library until the process exits); pageable or
 * page-locked host memory both work.  io->actions_dev must be NULL; every
 * other io field means what it does for sb_step_host.  Calls with more than
 * SB_NOALLOC_MAX_ENVS envs return SB_E_ARG, and so do calls whose records do
 * not live on the current device (the array used is the current device's).
 * The first call on a device looks up the array's device address
 * (cudaGetSymbolAddress) with that device current and keeps it until the
 * process exits; make that first call before any stream capture.  A
 * cudaDeviceReset (or anything else that tears down the device's primary
 * context) invalidates the kept address: do not call this entry point after
 * one.  Every call on a
 * device shares the one array: calls that overlap on the GPU (on different
 * streams) race on it.  Each call overwrites the entries it reads, so nothing
 * needs clearing between calls.  Nothing is allocated. */
#define SB_NOALLOC_MAX_ENVS 262144
int sb_step_host_noalloc(const sb_state *s, const sb_host_io *io, int64_t ply, const sb_policy *policy,
                         int auto_reset, const sb_step_out *out, void *stream);

/* ---- step server ----------------------------------------------------------
 * north-star: a persistent kernel that plays one fused ply (as sb_step with
 * the uniform policy, auto-reset and dense outputs) each time the host
 * publishes a step in a control block of mapped page-locked memory, so a
 * host-driven loop pays no kernel launch and no stream synchronisation per
 * ply.  Actions (or NULL: the cached proposals) are read from mapped
 * page-locked host memory; every output goes to device memory as in sb_step,
 * and after each step the CTA that completes it copies back_dev to the
 * mapped page-locked back_host before telling the host.  Every CTA gives up after limit_ns without a
 * step (status SB_STATUS_WAIT_TIMEOUT) and the kernel ends; nothing else may
 * use the state while the server runs.  At most (SMs x resident CTAs x 7)
 * envs (4,144 on a B200): all CTAs must be resident together. */
typedef struct sb_serve {
    int64_t *ctl;        /* mapped page-locked int64[17], zeroed by sb_serve_start: [0] step
                            published by the host, [1] stop, [16] last step every CTA finished */
    int64_t *dev;        /* device int64[4]: the kernel's relay of ctl (one CTA polls the host) */
    const void *back_dev;/* device range copied to back_host after every step, e.g. the out */
    void *back_host;     /*   fields reward / next_action / done laid out contiguously; mapped */
    int64_t back_bytes;  /*   page-locked; 16-byte aligned, a multiple of 16 bytes */
    int64_t n_ctas;      /* set by sb_serve_start */
    int64_t limit_ns;    /* longest a CTA waits for the next step (e.g. 2e9) */
} sb_serve;

int sb_serve_start(const sb_state *s, int64_t ply0, int auto_reset, const int64_t *actions_host,
                   const sb_step_out *out, sb_serve *sv, void *stream);
/* publish step t (1, 2, ...) and wait, at most timeout_ns, until every CTA has finished it */
int sb_serve_step(const sb_serve *sv, int64_t t, int64_t timeout_ns);
/* ask the kernel to stop after step t_done and wait for it on `stream` */
int sb_serve_stop(const sb_serve *sv, int64_t t_done, void *stream);

/* north-star: a trajectory ring of n_slots slots; every array is laid out
 * [n_slots, n, ...] and any pointer may be NULL. */
typedef struct sb_traj {
    void *infostate;           /* [T,n,C,10,10], see info_dtype / info_layout */
    int32_t info_dtype;
    int32_t info_layout;
    uint8_t *mask_u8;          /* [T,n,100,100] legal mask of the slot's state */
    uint8_t *mask_bits;        /* [T,n,1250] bit-packed legal mask of the slot's state */
    int16_t *action;           /* [T,n] action sampled at the slot's state (-1 when that
                                  state is a finished game, which no move leaves) */
    float *logprob;            /* [T,n] its log-prob under the policy */
    float *reward;             /* [T,n] player-0 reward of the slot's transition */
    uint8_t *done;             /* [T,n] the slot's transition ended the game */
    int64_t *hash;             /* [T,n] Zobrist hash of the slot's state */
    int64_t *stats;            /* [5] as sb_step_out.stats */
    int64_t n_slots;           /* T */
    int64_t slot0;             /* slot holding the current state */
} sb_traj;

/* north-star: n_plies plies in one launch, each env's record kept on chip.
 * n_plies == 0 observes the current state into slot slot0 (observation, mask,
 * sampled action and log-prob).  Ply p applies the action sampled for slot
 * (slot0+p) % T, writes reward / done there, auto-resets ended games when
 * auto_reset != 0, and writes the new state's observation, mask, sampled
 * action and log-prob into slot (slot0+p+1) % T.  The RNG ply of ply p is
 * ply + p. */
int sb_rollout(const sb_state *s, int64_t ply, const sb_policy *policy, int auto_reset, int32_t n_plies,
               const sb_traj *traj, void *stream);

/* north-star: belief resampling for search.  Sample env e becomes a copy of
 * root root_of[e] (roots: a state of n_roots envs) whose side-not-to-move has
 * its unrevealed identities re-dealt uniformly among the assignments
 * consistent with the side to move's information (moved pieces are never a
 * Bomb or the Flag).  Chase rings start empty; the hash is recomputed. */
int sb_belief_resample(const sb_state *roots, const sb_state *samples, const int64_t *root_of, void *stream);

/* north-star: sample an action for every env's current state at `ply`. */
int sb_sample_actions(const sb_state *s, int64_t ply, const sb_policy *policy, int64_t *actions, float *logprob,
                      void *stream);

/* ---- observations of the current state ---------------------------------- */
/* compute_legal_action_mask (csrc/stratego_buffer.cu:448-523, cpp:123-139):
 * [n,100,100] uint8 0/1. */
int sb_legal_mask_u8(const sb_state *s, uint8_t *mask, void *stream);
/* north-star: bit-packed [n,1250] variant. */
int sb_legal_mask_bits(const sb_state *s, uint8_t *bits, void *stream);
/* compute_infostate_tensor (csrc/stratego_buffer.cu:668-797, cpp:154-176). */
int sb_infostate(const sb_state *s, void *out, int dtype, int layout, void *stream);
/* hash_board (csrc/stratego_buffer.cu:805-845, cpp:189-203). */
int sb_hash_board(const sb_state *s, int64_t *out, void *stream);
/* get_has_legal_movement (csrc/stratego_buffer.cpp:216-219): [n] uint8. */
int sb_has_legal_movement(const sb_state *s, uint8_t *out, void *stream);

/* Getters of csrc/stratego_buffer.cpp:179-220 and the tracker state, written
 * in the reference's tensor layout.  Every pointer may be NULL. */
typedef struct sb_export {
    int8_t *board_owner;        /* [n,100] */
    int8_t *board_piece;        /* [n,100] */
    int8_t *current_player;     /* [n] */
    int8_t *outcome;            /* [n] */
    uint8_t *terminated;        /* [n] */
    uint8_t *flag_captured;     /* [n] */
    int32_t *move_number;       /* [n] */
    int32_t *moves_since_attack;/* [n] */
    int32_t *terminated_since;  /* [n] */
    uint8_t *moved_squares;     /* [n,100] */
    uint8_t *revealed_squares;  /* [n,100] */
    int32_t *move_history;      /* [n,32] */
    int32_t *move_history_head; /* [n] */
    int32_t *move_history_len;  /* [n] */
    int32_t *two_square_count;  /* [n,2] */
    int32_t *two_square_pair_lo;/* [n,2] */
    int32_t *two_square_pair_hi;/* [n,2] */
    uint8_t *two_square_violation; /* [n] */
    int32_t *chase_hash_head;   /* [n,2] */
    int32_t *chase_hash_len;    /* [n,2] */
    int32_t *chase_last_src;    /* [n,2] */
    uint8_t *chasing_violation; /* [n] */
    int32_t *episode;           /* [n] */
    int32_t *invalid_count;     /* [n] */
    float *reward;              /* [n] compute_reward_pl0 (cpp:142-151) */
    uint8_t *isf_two_square;    /* [n,100,6] SB_RULES_ISF per-square segment intersections (lo,hi)
                                   of the piece's last 1, 2, 3 moves, 255 = none */
    int8_t *isf_threats;        /* [n,2,4] squares each side's last move threatened, -1 = none */
    uint8_t *isf_evasion;       /* [n,2] each side's last move was an evasion */
} sb_export;

int sb_export_state(const sb_state *s, const sb_export *out, void *stream);

/* north-star: Σ move_number over envs into *out (current_step, cpp:301-303). */
int sb_sum_move_number(const sb_state *s, int64_t *out, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* STRATEGO_B200_H */
