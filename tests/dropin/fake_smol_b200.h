/*
 * fake_smol_b200.h -- the checking helpers of fake_smol_b200.c.
 */
#ifndef FAKE_SMOL_B200_H
#define FAKE_SMOL_B200_H

#include <stdio.h>

#include "device_decoder.h"

extern int g_failures;                     /* failed CHECKs (and frees of foreign pointers) */
extern int g_live, g_allocs, g_fail_at;    /* live allocations, allocations made, the one to fail */
extern int g_prefills, g_steps, g_check_embeds;
extern int g_fail_call;                    /* the next prefill / decode call fails after a partial write */
extern smol_b200_qkn_model g_last_model;   /* as passed to the last prefill / decode call */

#define CHECK(cond)                                                                   \
    do {                                                                              \
        if (!(cond)) {                                                                \
            fprintf(stderr, "%s:%d: check failed: %s\n", __FILE__, __LINE__, #cond); \
            g_failures++;                                                             \
        }                                                                             \
    } while (0)

/* bytes of the live allocation from p to its end (0 when p is not inside one) */
size_t dev_bytes_from(const void *p);
/* every weight of m is a live device allocation of sufficient size */
int model_on_device(const smol_b200_qkn_model *m);
uint16_t tag_k(int layer, int pos);
uint16_t tag_v(int layer, int pos);

#endif
