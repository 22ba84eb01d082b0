/* attn_bwd_b200.h — C ABI of the B200 (sm_100a) GQA attention-backward path.
 *
 * Replaces the hot path of the reference's
 *   custom_kernel((grad_attn_output, attn_weights, attn_weights_dropped,
 *                  value_states, dropout_mask, attention_dropout))
 *       -> (grad_attn_scores, grad_value_states)
 * (attn_bwd/starting_point.py:27-70; called by eval_modal_attn_bwd.py:273,339,381
 * and append.py:29-33).  Layout is fixed by the reference (starting_point.py:4-17):
 *
 *   grad_attn_output      dO   [bs, seq_q, 80, 128]      bf16
 *   attn_weights          P    [bs, 80, seq_q, seq_kv]   bf16
 *   attn_weights_dropped  Pd   [bs, 80, seq_q, seq_kv]   bf16
 *   value_states          V    [bs, 8, seq_kv, 128]      bf16
 *   dropout_mask          M    [bs, 80, seq_q, seq_kv]   bool (1 byte, 0 or 1)
 *   grad_attn_scores      dS   [bs, 80, seq_q, seq_kv]   bf16 (output)
 *   grad_value_states     dV   [bs, 8, seq_kv, 128]      bf16 (output)
 *
 * All pointers are device pointers to contiguous tensors, 16-byte aligned (the host-buffer
 * calls also take host pointers, named *_h).  Every call is asynchronous on `stream` and
 * returns 0 on success or one of the ATTN_BWD_E* codes (nothing is launched on error).
 *
 * Memory and resources: no call allocates device memory for tensors; outputs and (for the
 * host-buffer call) device buffers are the caller's.  The library does create, lazily and
 * per device, resources that live until attn_bwd_b200_release() or process exit:
 *   - on the first full call: one side stream (dV runs there next to dS) and two events;
 *   - on the second full call with a given argument list: an instantiated CUDA graph of
 *     that call's launches (a 16-entry LRU per device; a graph holds a little device
 *     memory for its nodes) and one private capture stream;
 *   - on the first host-buffer call: two copy streams and 130 events.
 * A device-side error word (see attn_bwd_b200_poll_error) is a static __device__ variable.
 */
#ifndef ATTN_BWD_B200_H
#define ATTN_BWD_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* attn_bwd_stream_t; /* == cudaStream_t */

enum {
  ATTN_BWD_OK = 0,
  ATTN_BWD_EINVAL = 1,       /* negative size, unit range outside [0, bs*8], null pointer */
  ATTN_BWD_EALIGN = 2,       /* a pointer is not 16-byte aligned */
  ATTN_BWD_EUNSUPPORTED = 3, /* shape has no kernel path */
  ATTN_BWD_ETMAP = 4,        /* TMA descriptor encoding failed */
  ATTN_BWD_ECUDA = 5,        /* a CUDA runtime call failed (launch, attribute query) */
  ATTN_BWD_EDEVICE = 6,      /* current device is not compute capability 10.x */
  ATTN_BWD_EKERNEL = 7       /* a kernel's bounded wait gave up (see attn_bwd_b200_poll_error) */
};

/* Full call: both outputs.  Replaces starting_point.py:27-70 (custom_kernel).
 * attention_dropout follows the reference: the mask and 1/(1-p) are applied
 * only when attention_dropout > 0 (starting_point.py:51-54). */
int attn_bwd_b200(const void* grad_attn_output, const void* attn_weights, const void* attn_weights_dropped,
                  const void* value_states, const uint8_t* dropout_mask, float attention_dropout, int bs,
                  int seq_q, int seq_kv, void* grad_attn_scores, void* grad_value_states,
                  attn_bwd_stream_t stream);

/* Sharded call over independent units u = b*8 + kv_head in [unit_begin, unit_end).
 * grad_attn_output and value_states are the FULL tensors; attn_weights,
 * attn_weights_dropped, dropout_mask, grad_attn_scores point at the first
 * element of head 10*unit_begin (i.e. [b0, 10*kvh0, 0, 0]) and hold
 * (unit_end-unit_begin)*10 heads; grad_value_states points at dV[unit_begin]
 * and holds (unit_end-unit_begin) [seq_kv,128] slabs.  Same math as
 * attn_bwd_b200 restricted to those units; the reference has no sharding, this
 * is the per-GPU call of the multi-GPU partition over batch x KV head. */
int attn_bwd_b200_shard(const void* grad_attn_output, const void* attn_weights, const void* attn_weights_dropped,
                        const void* value_states, const uint8_t* dropout_mask, float attention_dropout, int bs,
                        int seq_q, int seq_kv, int unit_begin, int unit_end, void* grad_attn_scores,
                        void* grad_value_states, attn_bwd_stream_t stream);

/* The two fused kernels alone (same sharding arguments), for timing and tests.
 * dS: starting_point.py:44-59.  dV: starting_point.py:61-68. */
int attn_bwd_b200_ds_shard(const void* grad_attn_output, const void* attn_weights, const void* value_states,
                           const uint8_t* dropout_mask, float attention_dropout, int bs, int seq_q, int seq_kv,
                           int unit_begin, int unit_end, void* grad_attn_scores, attn_bwd_stream_t stream);
int attn_bwd_b200_dv_shard(const void* grad_attn_output, const void* attn_weights_dropped, int bs, int seq_q,
                           int seq_kv, int unit_begin, int unit_end, void* grad_value_states,
                           attn_bwd_stream_t stream);

/* Full call without attn_weights_dropped.  The dV kernel forms each K chunk of P_drop in
 * shared memory as bf16(P * mask * 1/(1-p)) from the attn_weights and dropout_mask tiles it
 * streams, which is how the reference's inputs are made (eval_modal_attn_bwd.py:159-161:
 * attn_weights_dropped = bf16(attn_weights * mask / (1-p))).  Valid only for callers whose
 * P_drop is that product: it does NOT reproduce the reference for an arbitrary P_drop
 * (starting_point.py:62-64 reads the given tensor).  A caller using it never materialises
 * P_drop (2 bytes per score element of memory, and its host->device copy).  Requires
 * 0 <= attention_dropout < 1 (else ATTN_BWD_EINVAL) and seq_kv % 16 == 0 (else
 * ATTN_BWD_EUNSUPPORTED).  Sharding arguments as attn_bwd_b200_shard.  Replaces nothing in
 * the reference: it is the optional P_drop-free variant, behind its own entry point. */
int attn_bwd_b200_shard_from_mask(const void* grad_attn_output, const void* attn_weights, const void* value_states,
                                  const uint8_t* dropout_mask, float attention_dropout, int bs, int seq_q, int seq_kv,
                                  int unit_begin, int unit_end, void* grad_attn_scores, void* grad_value_states,
                                  attn_bwd_stream_t stream);

/* Host-buffer call: the same result as attn_bwd_b200_shard for inputs and outputs that live
 * in HOST memory, for callers whose tensors are not yet on the GPU.  The reference's
 * custom_kernel (starting_point.py:27-70) takes device tensors and has no such form; this
 * is the end-to-end call of the multi-GPU split with the host<->device copies included.
 *   *_h   host pointers with the shard layout of attn_bwd_b200_shard (dO_h and V_h whole,
 *         P_h / Pd_h / M_h / dS_h from head 10*unit_begin, dV_h from slab unit_begin);
 *         page-locked (cudaHostAlloc / pinned) memory lets the copies overlap; pageable
 *         memory works but the copies then serialise with the host thread.
 *   *_d   caller-allocated device buffers of the same sizes (16-byte aligned); the call
 *         allocates nothing.  On return from the stream they hold the inputs and outputs.
 *   chunks  pipeline depth: the unit range is cut into up to `chunks` pieces (0 = 16, at
 *         most 64) on boundaries that keep every slice 16-byte aligned; chunk k's
 *         host->device copies, kernels and device->host copies run on three streams, so the
 *         two copy directions and the kernels overlap.
 * Asynchronous on `stream`: all work starts after what is already queued there, and the
 * stream waits for the last device->host copy.  Calls on one device are serialised on
 * the host (the copy streams are per device). */
int attn_bwd_b200_host_shard(const void* grad_attn_output_h, const void* attn_weights_h,
                             const void* attn_weights_dropped_h, const void* value_states_h,
                             const uint8_t* dropout_mask_h, float attention_dropout, int bs, int seq_q,
                             int seq_kv, int unit_begin, int unit_end, void* grad_attn_scores_h,
                             void* grad_value_states_h, void* grad_attn_output_d, void* attn_weights_d,
                             void* attn_weights_dropped_d, void* value_states_d, uint8_t* dropout_mask_d,
                             void* grad_attn_scores_d, void* grad_value_states_d, int chunks,
                             attn_bwd_stream_t stream);
/* Host-buffer call over all bs*8 units (unit_begin = 0, unit_end = bs*8). */
int attn_bwd_b200_host(const void* grad_attn_output_h, const void* attn_weights_h,
                       const void* attn_weights_dropped_h, const void* value_states_h,
                       const uint8_t* dropout_mask_h, float attention_dropout, int bs, int seq_q, int seq_kv,
                       void* grad_attn_scores_h, void* grad_value_states_h, void* grad_attn_output_d,
                       void* attn_weights_d, void* attn_weights_dropped_d, void* value_states_d,
                       uint8_t* dropout_mask_d, void* grad_attn_scores_d, void* grad_value_states_d, int chunks,
                       attn_bwd_stream_t stream);

/* Synchronises the current device, returns the code a kernel's bounded wait
 * recorded since the last poll (0 if none) and clears it.  The reference's
 * evaluator has no counterpart; it reports exceptions (eval_modal_attn_bwd.py:294-302). */
int attn_bwd_b200_poll_error(void);

/* Self-test of failure detection (no reference counterpart): launches one warp
 * that waits on a barrier nothing will complete, with a limit of limit_us
 * microseconds (1..1000000).  The wait gives up, records code 0x7001 for
 * attn_bwd_b200_poll_error and the kernel exits; the context stays usable.
 * No GPU fault, trap or hang is involved. */
int attn_bwd_b200_selftest_wait_timeout(int limit_us, attn_bwd_stream_t stream);

/* Human-readable text for an ATTN_BWD_E* code (static storage). */
const char* attn_bwd_b200_strerror(int code);

/* ABI version of this library (major*100 + minor). */
int attn_bwd_b200_version(void);

/* Frees the lazily created per-device resources listed at the top of this file (side,
 * capture and copy streams, events, cached launch graphs) of the CURRENT device, after
 * synchronising it.  Later calls re-create what they need.  No reference counterpart. */
int attn_bwd_b200_release(void);

/* Measurement and test options (no reference counterpart).  Every option defaults to -1,
 * "automatic": the library then picks the kernel form measured fastest for the shape,
 * which is what production callers should use.  An option forces one choice instead, for
 * A/B measurements and for tests that must reach every kernel form.  Options are
 * process-wide, take effect from the next call, and invalidate cached launch graphs.
 * Forcing a form never changes the math, only which kernel computes it (the compact dS
 * form rounds the masked dP~ to bf16 before the softmax step, as noted in its kernel).
 * Returns ATTN_BWD_EINVAL for an unknown option. */
enum {
  ATTN_BWD_OPT_DS_MODE = 0,      /* 0 recompute, 1 resident, 2 TMEM-held P, 3 compact (where the shape allows) */
  ATTN_BWD_OPT_ROW_KIND = 1,     /* 1 per-row re-aligned (rows not 16-byte multiples), 2 class tiles (any rows) */
  ATTN_BWD_OPT_DS_CLUSTER = 2,   /* n CTAs per row (1..8) for the resident form, when the row fits */
  ATTN_BWD_OPT_L2_PREFETCH = 3,  /* 0/1: L2 prefetch of a CTA's next unit during pass 2 (aligned rows) */
  ATTN_BWD_OPT_L2_HINT = 4,      /* 0 off, 1 aligned rows (default), 2 also class-tile rows */
  ATTN_BWD_OPT_SPLIT = 5,        /* 0 plain / 1 split form of the dS + dV overlap */
  ATTN_BWD_OPT_DV_SMS = 6,       /* SMs given to dV in the split form */
  ATTN_BWD_OPT_SIDE_STREAM = 7,  /* 0: dS and dV back to back on the caller's stream */
  ATTN_BWD_OPT_GRAPH = 8,        /* 0: never replay full calls from cached CUDA graphs */
  ATTN_BWD_OPT_MAP_CACHE = 9,    /* 0: encode every TMA descriptor on every call */
  ATTN_BWD_OPT_COUNT = 10
};
int attn_bwd_b200_set_option(int option, int value);
/* Current value of an option (-1 = automatic), or -2 for an unknown option. */
int attn_bwd_b200_get_option(int option);

#ifdef __cplusplus
}
#endif
#endif /* ATTN_BWD_B200_H */
