/* A C host of the simulator, built only on include/stratego_b200.h and the
 * shared library: n games stepped for `plies` plies through sb_step_host with
 * actions and results in page-locked host memory (read and written in place
 * by the kernel).  The games form `groups` states over contiguous slices of
 * the same arrays (env_base = the slice's offset), each on its own stream and
 * stepped in turn, so one group's host turn overlaps the other groups' plies.
 * Ply 0 plays the device's proposals; every later ply plays, as host actions,
 * the proposals the previous ply returned.
 *
 * Writes to `out` (unless it is "-"): for every ply, reward f32[n], done
 * u8[n] and next_action i16[n]; then the final game records uint8[n,256].
 * Prints the time per step (every group's ply) after the first 10 plies.
 *
 * usage: c_host_loop n plies groups zobrist.bin out.bin|- */
#define _POSIX_C_SOURCE 199309L
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include <cuda_runtime.h>

#include "stratego_b200.h"

#define CK(x)                                                                      \
    do {                                                                           \
        cudaError_t e_ = (x);                                                      \
        if (e_ != cudaSuccess) {                                                   \
            fprintf(stderr, "%s: %s\n", #x, cudaGetErrorString(e_));               \
            return 1;                                                              \
        }                                                                          \
    } while (0)
#define SB(x)                                                                      \
    do {                                                                           \
        int rc_ = (x);                                                             \
        if (rc_ != SB_OK) {                                                        \
            fprintf(stderr, "%s: %d %s\n", #x, rc_, sb_last_error());              \
            return 1;                                                              \
        }                                                                          \
    } while (0)

enum { MAX_GROUPS = 16, ZOB_N = 10 * 10 * 2 * 13 };

static double now_s(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return ts.tv_sec + 1e-9 * ts.tv_nsec;
}

int main(int argc, char **argv) {
    if (argc != 6) {
        fprintf(stderr, "usage: %s n plies groups zobrist.bin out.bin|-\n", argv[0]);
        return 2;
    }
    const int64_t n = atoll(argv[1]);
    const int plies = atoi(argv[2]), G = atoi(argv[3]);
    const int log = strcmp(argv[5], "-") != 0;
    const uint64_t seed = 7;
    const int64_t P = 4096, INFO = (int64_t)SB_NUM_CHANNELS * 100 * 2; /* bf16 dense */
    if (n < G || G < 1 || G > MAX_GROUPS || plies < 1) return 2;

    static int64_t zob[ZOB_N];
    FILE *zf = fopen(argv[4], "rb");
    if (!zf || fread(zob, sizeof zob, 1, zf) != 1) return 2;
    fclose(zf);

    uint8_t *rec, *pool, *mask, *info;
    int64_t *ring, *dzob;
    int32_t *status, h_status = 0;
    CK(cudaMalloc((void **)&rec, n * SB_RECORD_BYTES));
    CK(cudaMalloc((void **)&ring, n * 2 * 64 * sizeof(int64_t)));
    CK(cudaMalloc((void **)&dzob, sizeof zob));
    CK(cudaMalloc((void **)&pool, P * 40));
    CK(cudaMalloc((void **)&status, sizeof(int32_t)));
    CK(cudaMalloc((void **)&mask, n * 10000));
    CK(cudaMalloc((void **)&info, n * INFO));
    CK(cudaMemcpy(dzob, zob, sizeof zob, cudaMemcpyHostToDevice));
    CK(cudaMemset(status, 0, sizeof(int32_t)));
    CK(cudaMemset(info, 0, n * INFO)); /* the zero planes 43-455, written once */
    float *reward;
    uint8_t *done;
    int16_t *next;
    int64_t *acts;
    CK(cudaHostAlloc((void **)&reward, n * sizeof(float), cudaHostAllocMapped));
    CK(cudaHostAlloc((void **)&done, n, cudaHostAllocMapped));
    CK(cudaHostAlloc((void **)&next, n * sizeof(int16_t), cudaHostAllocMapped));
    CK(cudaHostAlloc((void **)&acts, n * sizeof(int64_t), cudaHostAllocMapped));
    SB(sb_make_setup_pool(seed, 0, P, pool, NULL));
    CK(cudaDeviceSynchronize());

    /* per-ply logs of the results (the host's copy, taken in each group's turn) */
    float *l_rew = log ? malloc((size_t)plies * n * sizeof(float)) : NULL;
    uint8_t *l_done = log ? malloc((size_t)plies * n) : NULL;
    int16_t *l_next = log ? malloc((size_t)plies * n * sizeof(int16_t)) : NULL;
    if (log && (!l_rew || !l_done || !l_next)) return 1;

    sb_state st[MAX_GROUPS];
    sb_step_out out[MAX_GROUPS];
    sb_host_io io[MAX_GROUPS];
    cudaStream_t stream[MAX_GROUPS];
    int64_t off[MAX_GROUPS], cnt[MAX_GROUPS];
    const sb_policy pol = {SB_POLICY_UNIFORM, 0, NULL};
    for (int g = 0; g < G; ++g) {
        const int64_t q = n / G, r = n % G;
        cnt[g] = q + (g < r ? 1 : 0);
        off[g] = g * q + (g < r ? g : r);
        const int64_t o = off[g];
        const sb_state s = {rec + o * SB_RECORD_BYTES, ring + o * 2 * 64, dzob, pool, P, cnt[g], o, seed,
                            100, 4000, 3, SB_RULES_CUDA, status, NULL};
        st[g] = s;
        memset(&out[g], 0, sizeof out[g]);
        out[g].mask_u8 = mask + o * 10000;
        out[g].infostate = info + o * INFO;
        out[g].info_dtype = SB_DTYPE_BF16;
        out[g].info_layout = SB_LAYOUT_DENSE_LIVE;
        out[g].reward = reward + o;
        out[g].done = done + o;
        out[g].next_action = next + o;
        memset(&io[g], 0, sizeof io[g]);
        io[g].actions_host = NULL; /* ply 0: the device's proposals */
        io[g].sync = 0;
        CK(cudaStreamCreate(&stream[g]));
        SB(sb_init_state(&st[g], stream[g]));
        SB(sb_reset_pool(&st[g], 1, stream[g]));
    }

    const int warm = plies > 20 ? 10 : 0;
    double t0 = now_s();
    for (int g = 0; g < G; ++g) SB(sb_step_host(&st[g], &io[g], 0, &pol, 1, &out[g], stream[g]));
    for (int t = 0; t < plies; ++t) {
        if (t == warm) t0 = now_s();
        for (int g = 0; g < G; ++g) {
            CK(cudaStreamSynchronize(stream[g]));
            const int64_t a = off[g], b = off[g] + cnt[g];
            if (log) {
                memcpy(l_rew + (size_t)t * n + a, reward + a, (b - a) * sizeof(float));
                memcpy(l_done + (size_t)t * n + a, done + a, b - a);
                memcpy(l_next + (size_t)t * n + a, next + a, (b - a) * sizeof(int16_t));
            }
            if (t + 1 == plies) continue;
            for (int64_t i = a; i < b; ++i) acts[i] = next[i]; /* the host policy: play the proposals */
            io[g].actions_host = acts + a;
            SB(sb_step_host(&st[g], &io[g], t + 1, &pol, 1, &out[g], stream[g]));
        }
    }
    const double dt = now_s() - t0;
    CK(cudaDeviceSynchronize());
    CK(cudaMemcpy(&h_status, status, sizeof h_status, cudaMemcpyDeviceToHost));
    printf("c_host_loop n=%lld groups=%d: %.2f us per step, %.1f M updates/s, status %d\n", (long long)n, G,
           1e6 * dt / (plies - warm), 1e-6 * n * (plies - warm) / dt, h_status);

    if (log) {
        uint8_t *h_rec = malloc(n * SB_RECORD_BYTES);
        if (!h_rec) return 1;
        CK(cudaMemcpy(h_rec, rec, n * SB_RECORD_BYTES, cudaMemcpyDeviceToHost));
        FILE *of = fopen(argv[5], "wb");
        if (!of) return 2;
        for (int t = 0; t < plies; ++t) {
            fwrite(l_rew + (size_t)t * n, sizeof(float), n, of);
            fwrite(l_done + (size_t)t * n, 1, n, of);
            fwrite(l_next + (size_t)t * n, sizeof(int16_t), n, of);
        }
        fwrite(h_rec, SB_RECORD_BYTES, n, of);
        fclose(of);
        free(h_rec);
    }
    return h_status == 0 ? 0 : 1;
}
