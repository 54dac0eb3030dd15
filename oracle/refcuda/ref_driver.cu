// ref_driver.cu -- C ABI over the reference's own CUDA launchers -- TEST
// INFRASTRUCTURE.
//
// Built together with the reference's csrc/stratego_buffer.cu (compiled from
// its own source file, with the shim header beside this file standing in for
// the one c10 macro it uses) into oracle/_ref/libref_stratego_cuda.so.  Only
// tests/, tests/golden/make_golden_refcuda.py and bench.py's reference-CUDA
// timing load it: it runs the reference's kernels so that this repository's
// kernels can be checked against them and timed beside them.  Nothing in the
// product (ataraxos_b200/) links or calls it.
//
// Each entry point forwards plain device pointers to one launcher declared in
// csrc/stratego_buffer.cuh (:72-267) and returns 0, or the CUDA error code of
// the launch.  The state arrays are the reference class's tensors
// (csrc/stratego_buffer.cpp:24-55) in the same layout; the host-side parts of
// its methods (flag counts, masks, memsets) are restated with torch in
// oracle/refcuda.py.
#include <cuda_runtime.h>
#include <stdint.h>

#include "stratego_buffer.cuh"

extern "C" {

// Device pointers of the reference class's state (csrc/stratego_buffer.cpp:308-336).
typedef struct ref_state {
    int8_t *board_owner, *board_piece;                        // [N,10,10]
    int8_t *current_player;                                   // [N]
    int32_t *move_number, *moves_since_attack;                // [N]
    int8_t *outcome;                                          // [N]
    uint8_t *terminated;                                      // [N] bool
    uint8_t *moved_squares, *revealed_squares;                // [N,100] bool
    int32_t *move_history, *move_history_head, *move_history_len;  // [N,32], [N], [N]
    int32_t *two_square_count, *two_square_pair_lo, *two_square_pair_hi;  // [N,2]
    uint8_t *two_square_violation;                            // [N] bool
    const int64_t *zobrist_table;                             // [10,10,2,13]
    int64_t *chase_hashes;                                    // [N,2,64]
    int32_t *chase_hash_head, *chase_hash_len, *chase_last_src;  // [N,2]
    uint8_t *chasing_violation;                               // [N] bool
    int32_t n;
} ref_state;

static int last_error() { return (int)cudaGetLastError(); }

int ref_hello_world(int *out, void *stream) {
    stratego::launch_hello_world(out, 1, (cudaStream_t)stream);
    return last_error();
}

int ref_apply_actions(const ref_state *s, const int64_t *actions, void *stream) {
    stratego::launch_apply_actions(
        s->board_owner, s->board_piece, actions, s->current_player, s->move_number, s->moves_since_attack,
        s->outcome, (bool *)s->terminated, (bool *)s->moved_squares, (bool *)s->revealed_squares, s->move_history,
        s->move_history_head, s->move_history_len, s->two_square_count, s->two_square_pair_lo,
        s->two_square_pair_hi, (bool *)s->two_square_violation, s->zobrist_table, s->chase_hashes,
        s->chase_hash_head, s->chase_hash_len, s->chase_last_src, (bool *)s->chasing_violation, s->n,
        (cudaStream_t)stream);
    return last_error();
}

int ref_legal_action_mask(const ref_state *s, uint8_t *mask, void *stream) {
    stratego::launch_legal_action_mask(s->board_owner, s->board_piece, s->current_player, (bool *)mask, s->n,
                                       (cudaStream_t)stream);
    return last_error();
}

int ref_reset(const ref_state *s, const int8_t *setup_red, const int8_t *setup_blue, void *stream) {
    stratego::launch_reset(
        s->board_owner, s->board_piece, setup_red, setup_blue, s->current_player, s->move_number,
        s->moves_since_attack, s->outcome, (bool *)s->terminated, (bool *)s->moved_squares,
        (bool *)s->revealed_squares, s->move_history, s->move_history_head, s->move_history_len,
        s->two_square_count, s->two_square_pair_lo, s->two_square_pair_hi, (bool *)s->two_square_violation,
        s->chase_hashes, s->chase_hash_head, s->chase_hash_len, s->chase_last_src, (bool *)s->chasing_violation,
        s->n, (cudaStream_t)stream);
    return last_error();
}

int ref_infostate(const ref_state *s, float *out, void *stream) {
    stratego::launch_compute_infostate(s->board_owner, s->board_piece, s->current_player, s->move_number,
                                       s->moves_since_attack, (const bool *)s->moved_squares,
                                       (const bool *)s->revealed_squares, s->move_history, s->move_history_head,
                                       s->move_history_len, out, s->n, (cudaStream_t)stream);
    return last_error();
}

int ref_hash_board(const ref_state *s, int64_t *out, void *stream) {
    stratego::launch_hash_board(s->board_owner, s->board_piece, s->zobrist_table, out, s->n, (cudaStream_t)stream);
    return last_error();
}

}  // extern "C"
