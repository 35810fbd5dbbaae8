/* bccl_c_example: the C interface from plain C11 (no C++ in the caller).
 *
 *   bccl_run -np 4 bccl_c_example
 *
 * Each rank gets its rank from BCCL_RANK / BCCL_WORLD_SIZE; rank 0 creates the unique id and
 * writes "ip:port" to BCCL_ID_FILE (or every rank uses BCCL_MASTER when it is set), then every
 * rank runs an int32 AllReduce (SUM), a grouped AllGather + ReduceScatter (AVG) and a
 * Send/Recv around the ring on host memory, checks the results and prints one line. */
#define _POSIX_C_SOURCE 200809L /* nanosleep under -std=c11 */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>
#include <unistd.h>

#include "bccl/c_api.h"

static int fail(const char* what) {
    fprintf(stderr, "bccl_c_example: %s: %s\n", what, bcclGetLastError());
    return 1;
}

static int read_id(const char* path, bcclConfig* cfg) {
    for (int i = 0; i < 6000; ++i) { /* up to 60 s */
        FILE* f = fopen(path, "r");
        if (f != NULL) {
            char buf[128] = {0};
            size_t n = fread(buf, 1, sizeof(buf) - 1, f);
            fclose(f);
            char* colon = strrchr(buf, ':');
            if (n > 0 && colon != NULL) {
                *colon = '\0';
                snprintf(cfg->ip_addr, sizeof(cfg->ip_addr), "%s", buf);
                cfg->port = (uint16_t)atoi(colon + 1);
                return 0;
            }
        }
        struct timespec ts = {0, 10 * 1000 * 1000};
        nanosleep(&ts, NULL);
    }
    return 1;
}

int main(void) {
    const char* rank_s = getenv("BCCL_RANK");
    const char* world_s = getenv("BCCL_WORLD_SIZE");
    const char* path = getenv("BCCL_ID_FILE");
    const char* master = getenv("BCCL_MASTER");
    if (rank_s == NULL || world_s == NULL || (path == NULL && master == NULL)) {
        fprintf(stderr, "run under bccl_run\n");
        return 2;
    }
    bcclConfig cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.rank = atoi(rank_s);
    cfg.world_size = atoi(world_s);
    cfg.device = -1;
    cfg.n_channels = 2;
    bcclComm_t comm = NULL;
    if (bcclCommCreate(&comm) != 0) return fail("create");
    if (cfg.rank == 0) {
        if (bcclGetUniqueId(comm, cfg.ip_addr, &cfg.port) != 0) return fail("unique id");
        if (master == NULL) {
            char tmp[4096];
            snprintf(tmp, sizeof(tmp), "%s.tmp", path);
            FILE* f = fopen(tmp, "w");
            if (f == NULL) return fail("id file");
            fprintf(f, "%s:%u", cfg.ip_addr, (unsigned)cfg.port);
            fclose(f);
            if (rename(tmp, path) != 0) return fail("id file rename");
        }
    } else if (master != NULL) {
        const char* colon = strrchr(master, ':');
        if (colon == NULL) return 2;
        snprintf(cfg.ip_addr, sizeof(cfg.ip_addr), "%.*s", (int)(colon - master), master);
        cfg.port = (uint16_t)atoi(colon + 1);
    } else if (read_id(path, &cfg) != 0) {
        return fail("waiting for the unique id");
    }
    if (bcclCommInit(comm, &cfg) != 0) return fail("init");
    const int r = cfg.rank, n = cfg.world_size;
    int bad = 0;

    enum { kCount = 1000 };
    int32_t x[kCount], y[kCount];
    for (int i = 0; i < kCount; ++i) x[i] = r * 7 + i;
    if (bcclAllReduce(comm, x, y, kCount, bcclInt32, bcclSum, 1.0f, 0, 0, 0) != 0) return fail("allreduce");
    for (int i = 0; i < kCount; ++i) bad += y[i] != 7 * n * (n - 1) / 2 + n * i;

    float* g = malloc(sizeof(float) * 64 * (size_t)n);
    float* rs_in = malloc(sizeof(float) * 64 * (size_t)n);
    float mine[64], shard[64];
    for (int i = 0; i < 64; ++i) mine[i] = (float)(r + i);
    for (int i = 0; i < 64 * n; ++i) rs_in[i] = (float)(r * 2);
    bcclGroupStart(comm);
    if (bcclAllGather(comm, mine, g, 64, bcclFloat32, 0, 0) != 0) return fail("allgather");
    if (bcclReduceScatter(comm, rs_in, shard, 64, bcclFloat32, bcclAvg, 0, 0) != 0) return fail("reducescatter");
    if (bcclGroupEnd(comm, 0, 0) != 0) return fail("group");
    for (int q = 0; q < n; ++q)
        for (int i = 0; i < 64; ++i) bad += g[q * 64 + i] != (float)(q + i);
    for (int i = 0; i < 64; ++i) bad += shard[i] != (float)(n - 1); /* mean of 2q over q */

    if (n > 1) {
        int32_t s[16], got[16];
        for (int i = 0; i < 16; ++i) s[i] = 100 * r + i;
        bcclGroupStart(comm);
        bcclSend(comm, s, 16, bcclInt32, (r + 1) % n, 0, 0);
        bcclRecv(comm, got, 16, bcclInt32, (r + n - 1) % n, 0, 0);
        if (bcclGroupEnd(comm, 0, 0) != 0) return fail("send/recv");
        for (int i = 0; i < 16; ++i) bad += got[i] != 100 * ((r + n - 1) % n) + i;
    }
    free(g);
    free(rs_in);
    bcclCommFinalize(comm);
    bcclCommDestroy(comm);
    printf("rank %d of %d: %s\n", r, n, bad ? "FAILED" : "ok");
    return bad ? 1 : 0;
}
