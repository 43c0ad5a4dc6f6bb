/*
 * axtp.h — C ABI of the tensor-parallel sum over NVLink peer memory.
 *
 * The all-reduce that the decode step runs after its row-split products
 * (axdec.h, kind 2 of axdec_tp_allreduce_kind), for callers that manage their
 * own buffers: every rank passes the same group, with the other ranks' buffers
 * mapped into its address space (CUDA IPC or any peer mapping).  Replaces the
 * NCCL all-reduce wrapper of the tensor-parallel plan (ax_allreduce_sum);
 * the reference itself runs on one CPU and has no collective.
 *
 * Same conventions as axq8.h: plain C, status codes, axq8_last_error().
 */
#ifndef AXION_B200_AXTP_H
#define AXION_B200_AXTP_H

#include <stdint.h>

#include "axq8_status.h"

#ifdef __cplusplus
extern "C" {
#endif

#define AXTP_MAX_RANKS 8

typedef struct axtp_group {
    float* part[AXTP_MAX_RANKS];     /* every rank's partial [n] fp32, as mapped here */
    float* out[AXTP_MAX_RANKS];      /* every rank's output [n] fp32 */
    uint32_t* flags[AXTP_MAX_RANKS]; /* every rank's flags [2 * AXTP_MAX_RANKS], zero at start */
    uint32_t* epoch;                 /* this rank's counter, zero at start (local) */
    int32_t* ctas_done;              /* this rank's counter, zero at start (local) */
    int32_t rank, world;             /* 2 <= world <= AXTP_MAX_RANKS */
} axtp_group_t;

/* out[r] = sum over ranks of part (n % 4 == 0, 16-byte aligned buffers), on
 * every rank r, bit-identical on all ranks: rank r sums slice r in rank order
 * and writes it to every rank.  Collective: all `world` ranks call it with the
 * same n, in the same order, on their own GPU, concurrently.  Each wait on a
 * peer is bounded (about two seconds); on timeout the device status word
 * (axq8_status_read) becomes AXQ8_ERR_WAIT_TIMEOUT and the call's sums are
 * invalid.  Calls on one group must not overlap. */
int axtp_allreduce_sum(const axtp_group_t* g, int64_t n, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* AXION_B200_AXTP_H */
