/* A stand-in for libnccl for the failure tests of the data-parallel open (plamo_open_broadcast's
 * communicator setup, plamo_debug_nccl_init): the entry points libplamo_cuda loads, with the
 * behaviour FAKE_NCCL_MODE selects, and a count of the communicators handed out and taken back,
 * rewritten to FAKE_NCCL_LOG ("created destroyed aborted") after every change.
 *   ok     setup completes after a few polls of ncclCommGetAsyncError
 *   never  setup stays in progress forever (a peer that never joins)
 *   error  ncclCommInitRankConfig fails at once with ncclSystemError
 * It needs no GPU and opens no connection. */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

typedef struct { char internal[128]; } fake_uid;

enum { FAKE_SUCCESS = 0, FAKE_SYSTEM_ERROR = 2, FAKE_INVALID = 4, FAKE_IN_PROGRESS = 7 };

static int created, destroyed, aborted, polls;

static const char* mode(void) {
    const char* m = getenv("FAKE_NCCL_MODE");
    return m ? m : "ok";
}

static void record(void) {
    const char* path = getenv("FAKE_NCCL_LOG");
    if (!path) return;
    FILE* f = fopen(path, "w");
    if (!f) return;
    fprintf(f, "%d %d %d\n", created, destroyed, aborted);
    fclose(f);
}

int ncclGetUniqueId(fake_uid* id) {
    memset(id, 0x5a, sizeof(*id));
    return FAKE_SUCCESS;
}

int ncclCommInitRankConfig(void** comm, int nranks, fake_uid id, int rank, void* config) {
    (void)id;
    (void)config;
    if (!comm || nranks < 1 || rank < 0 || rank >= nranks) return FAKE_INVALID;
    if (strcmp(mode(), "error") == 0) return FAKE_SYSTEM_ERROR;
    *comm = malloc(64);
    created++;
    polls = 0;
    record();
    return FAKE_IN_PROGRESS;
}

int ncclCommInitRank(void** comm, int nranks, fake_uid id, int rank) {
    const int e = ncclCommInitRankConfig(comm, nranks, id, rank, NULL);
    return e == FAKE_IN_PROGRESS ? FAKE_SUCCESS : e;
}

int ncclCommGetAsyncError(void* comm, int* state) {
    if (!comm || !state) return FAKE_INVALID;
    if (strcmp(mode(), "never") == 0) {
        *state = FAKE_IN_PROGRESS;
    } else {
        *state = ++polls >= 3 ? FAKE_SUCCESS : FAKE_IN_PROGRESS;
    }
    return FAKE_SUCCESS;
}

int ncclCommAbort(void* comm) {
    free(comm);
    aborted++;
    record();
    return FAKE_SUCCESS;
}

int ncclCommDestroy(void* comm) {
    free(comm);
    destroyed++;
    record();
    return FAKE_SUCCESS;
}

int ncclBroadcast(const void* send, void* recv, size_t count, int type, int root, void* comm, void* stream) {
    (void)send; (void)recv; (void)count; (void)type; (void)root; (void)comm; (void)stream;
    return FAKE_SUCCESS;
}

const char* ncclGetErrorString(int e) {
    return e == FAKE_SYSTEM_ERROR ? "unhandled system error (fake)" : "fake NCCL error";
}
