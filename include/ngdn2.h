/*
 * ngdn2.h -- C ABI of the B200-native nested Gated DeltaNet (nested GDN-2)
 * forward hot path.
 *
 * Every entry point takes plain pointers, sizes and strides, returns 0 or a
 * negative NGDN2_ERR_* code, never throws, and never allocates, frees or
 * retains device memory: the caller passes every input, output and
 * workspace buffer. Launches go on the caller's CUDA stream (a cudaStream_t
 * passed as void*; NULL is the legacy default stream). No entry point
 * synchronises the stream.
 *
 * The entry points replace these functions of the reference project
 * (awehrs/nested_recurrent_memory, paths within that project):
 *
 *   ngdn2_fwd            nested_gdn2/ops/chunk.py:159-304  chunk_nested_gdn2_fwd
 *                        (and the forward of chunk_nested_gdn2, chunk.py:722-766,
 *                        whose Function.forward calls it, chunk.py:571-648)
 *   ngdn2_update_state   nested_gdn2/ops/update_fwd.py:131-204  update_state
 *   ngdn2_step           nested_gdn2/ops/naive.py:42-134  naive_step_nested_gdn2
 *                        (the one-token decode step the layer runs past the
 *                        chunked prefix, nested_gdn2.py:218-224)
 *
 * Layouts are the reference's (chunk.py:184-217): per-token tensors
 * [B, T, H, ...], states [B, H, L, K, V] float32, parameters
 * [L-1, H, ...] contiguous.
 */
#ifndef NGDN2_H_
#define NGDN2_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define NGDN2_API __attribute__((visibility("default")))
#else
#define NGDN2_API
#endif

#define NGDN2_ABI_VERSION 2
#define NGDN2_MAX_LEVELS 8
#define NGDN2_CHUNK 64

/* Element types of the floating-point tensors. */
enum {
  NGDN2_F32 = 0,
  NGDN2_BF16 = 1,
  NGDN2_F16 = 2
};

/* Promotion arms, the keys of the reference's PROBES registry
 * (nested_gdn2/ops/probe.py:139-142). */
enum {
  NGDN2_PROMOTION_LEARNED = 0, /* probe.py:69-102 */
  NGDN2_PROMOTION_MERGE = 1    /* probe.py:105-136 */
};

/* Kernel families. AUTO picks a tensor-core family when the shape and dtype
 * allow (K = V = 128, 16-bit q/k/v/b/w/o): the fused one-pass family for
 * L <= 3 with many (batch, head) pairs, else the level-segmented family;
 * otherwise the CUDA-core fp32 family. */
enum {
  NGDN2_PATH_AUTO = 0,
  NGDN2_PATH_SIMT = 1,   /* CUDA-core kernels, fp32 arithmetic throughout */
  NGDN2_PATH_TC = 2,     /* tcgen05 kernels, one fused scan per (batch, head); L <= 3 */
  NGDN2_PATH_TC_SEG = 3  /* tcgen05 kernels, every level a segmented scan (compose, combine,
                            replay) so few (batch, head) pairs still fill the GPU; any L */
};

/* Return codes. The Python host layer maps each to the reference's
 * ValueError message. */
enum {
  NGDN2_OK = 0,
  NGDN2_ERR_CHUNK_SIZE = -1,    /* chunk.py:230-231 "chunk_size must be 64" */
  NGDN2_ERR_N_POW2 = -2,        /* update_fwd.py:162-163 "power of two >= 16" */
  NGDN2_ERR_BLOCK_V = -3,       /* update_fwd.py:164-165 "block_v must be ..." */
  NGDN2_ERR_DIVISIBLE = -4,     /* update_fwd.py:166-167 "must be divisible" */
  NGDN2_ERR_UNIT_STRIDE = -5,   /* update_fwd.py:168-169 "unit-stride" */
  NGDN2_ERR_INCONSISTENT = -6,  /* update_fwd.py:170-171 "inconsistent" */
  NGDN2_ERR_SHAPE = -7,         /* a size out of the supported range */
  NGDN2_ERR_DTYPE = -8,         /* unknown dtype code */
  NGDN2_ERR_NULL = -9,          /* a required pointer is NULL */
  NGDN2_ERR_WORKSPACE = -10,    /* workspace smaller than ngdn2_fwd_workspace_size */
  NGDN2_ERR_UNSUPPORTED = -11,  /* requested path cannot run this shape/dtype */
  NGDN2_ERR_CUDA = -12,         /* a CUDA runtime call failed */
  NGDN2_ERR_ABI = -13,          /* abi_version mismatch */
  NGDN2_ERR_FIRING = -14        /* firing intervals not nested or not >= 1 */
};

/* Arguments of ngdn2_fwd. */
typedef struct ngdn2_fwd_args {
  int32_t abi_version;  /* NGDN2_ABI_VERSION */
  int32_t path;         /* NGDN2_PATH_* */
  int32_t B, T, H, K, V, L;
  int32_t chunk_size;   /* must be 64 (chunk.py:230-231) */
  int32_t promotion;    /* NGDN2_PROMOTION_* */
  int32_t dtype;        /* element type of the output o */
  int32_t param_dtype;  /* of query_banks and the four projections */
  float scale;          /* read scale; the reference default is K^-1/2 */
  int32_t n_max;        /* query_banks.shape[2] (N_MAX) */
  int32_t n_queries[NGDN2_MAX_LEVELS]; /* [l-1] = pairs for level l >= 1 */
  int32_t firing[NGDN2_MAX_LEVELS];    /* [l] = interval of level l in chunks; [0] == 1 */

  /* Per-token inputs: pointer, element type (NGDN2_F32/BF16/F16) and
   * element strides. Any strides are accepted, including 0 (broadcast); the
   * tensor-core path additionally wants unit-stride last dimensions. */
  const void* q;   int32_t q_dtype;   int64_t q_stride[5];   /* [B, T, H, L, K] */
  const void* k;   int32_t k_dtype;   int64_t k_stride[4];   /* [B, T, H, K] */
  const void* v;   int32_t v_dtype;   int64_t v_stride[4];   /* [B, T, H, V] */
  const void* g;   int32_t g_dtype;   int64_t g_stride[4];   /* [B, T, H, K] level-0 log-decay */
  const void* b;   int32_t b_dtype;   int64_t b_stride[4];   /* [B, T, H, K] level-0 erase gate */
  const void* w;   int32_t w_dtype;   int64_t w_stride[4];   /* [B, T, H, V] level-0 write gate */
  const void* mix; int32_t mix_dtype; int64_t mix_stride[4]; /* [B, T, H, L] read-mix weights */

  const void* query_banks;      /* [L-1, H, n_max, K] contiguous */
  const void* key_projections;  /* [L-1, H, K, V] */
  const void* b_projections;    /* [L-1, H, V, K] */
  const void* w_projections;    /* [L-1, H, V, V] */
  const void* g_projections;    /* [L-1, H, V, K] */

  const float* initial_state;   /* [B, H, L, K, V] or NULL for zeros */
  void* o;                      /* [B, T, H, V] contiguous, element type dtype */
  float* final_state;           /* [B, H, L, K, V] contiguous, always written */

  void* workspace;              /* device scratch, >= ngdn2_fwd_workspace_size */
  size_t workspace_bytes;
  int32_t* status;              /* optional device word; kernels OR in NGDN2_STATUS_* */

  /* Optional start gate: a device-visible word (device memory or mapped
   * pinned host memory) that a producer sets nonzero once the inputs are in
   * place. When non-NULL, the forward's first kernel polls it at most
   * gate_polls times (0 means 2^24) before any other work; if it is still
   * zero, NGDN2_STATUS_GATE_TIMEOUT is set in *status (status must then be
   * non-NULL) and every kernel of this forward returns without touching the
   * outputs. Lets a caller enqueue the forward before a host or peer
   * producer has finished writing its inputs, with a bounded wait instead
   * of a hang. */
  const volatile int32_t* gate;
  uint32_t gate_polls;
} ngdn2_fwd_args;

/* Device status bits (written to ngdn2_fwd_args.status when non-NULL). The
 * word is sticky: kernels only OR bits in; the caller clears it. */
enum {
  NGDN2_STATUS_WAIT_TIMEOUT = 1, /* a bounded pipeline wait gave up: outputs are not valid, and
                                    the CUDA context should be treated as suspect (an MMA or copy
                                    the wait was for may still have been in flight) */
  NGDN2_STATUS_GATE_TIMEOUT = 2  /* the start gate stayed zero: nothing was computed */
};

/* Arguments of ngdn2_update_state (update_fwd.py:131-204). */
typedef struct ngdn2_update_args {
  int32_t abi_version;
  int32_t B, NF, NG, H, K, V, N;
  int32_t block_v;      /* columns per program in the reference; validated the same way */
  int32_t dtype;        /* of keys, values, b, w */
  int32_t g_dtype;      /* of g */
  const void* keys;   int64_t keys_stride[5];   /* [B, NF, H, N, K] element strides; the K stride must be 1 */
  const void* values;                           /* [B, NF, H, N, V] contiguous */
  const void* g;                                /* [B, NF, H, K] contiguous */
  const void* b;                                /* [B, NF, H, N, K] contiguous */
  const void* w;                                /* [B, NF, H, N, V] contiguous */
  const float* initial_state;                   /* [B, H, K, V] or NULL */
  float* states;                                /* [B, NG, H, K, V] out */
  float* final_state;                           /* [B, H, K, V] out */
} ngdn2_update_args;

/* Arguments of ngdn2_update_state_bwd (update_bwd.py:167-263,
 * update_state_bwd): the gradients of sum(states * d_states) +
 * sum(final * d_final) for the write scan, fp32 outputs. */
typedef struct ngdn2_update_bwd_args {
  int32_t abi_version;
  int32_t B, NF, NG, H, K, V, N;
  int32_t block_v;      /* validated as in the forward; the kernel does not split V */
  int32_t dtype;        /* of keys, values, b, w */
  int32_t g_dtype;      /* of g */
  int32_t has_init;     /* write dinit */
  const float* states;                          /* [B, NG, H, K, V] from the forward */
  const void* keys;   int64_t keys_stride[5];   /* [B, NF, H, N, K]; the K stride must be 1 */
  const void* values;                           /* [B, NF, H, N, V] contiguous */
  const void* g;                                /* [B, NF, H, K] contiguous */
  const void* b;                                /* [B, NF, H, N, K] contiguous */
  const void* w;                                /* [B, NF, H, N, V] contiguous */
  const float* d_states;                        /* [B, NG, H, K, V] contiguous */
  const float* d_final;                         /* [B, H, K, V] contiguous */
  float* dkeys;                                 /* [B, NF, H, N, K] out */
  float* dvalues;                               /* [B, NF, H, N, V] out */
  float* dg;                                    /* [B, NF, H, K] out */
  float* db;                                    /* [B, NF, H, N, K] out */
  float* dw;                                    /* [B, NF, H, N, V] out */
  float* dinit;                                 /* [B, H, K, V] out, or NULL */
  void* workspace;                              /* >= ngdn2_update_bwd_workspace_size */
  size_t workspace_bytes;
} ngdn2_update_bwd_args;

/* Arguments of ngdn2_step: one token of every batch row (naive.py:42-134).
 * Per-token inputs carry no T dimension. */
typedef struct ngdn2_step_args {
  int32_t abi_version;
  int32_t B, H, K, V, L;
  int32_t chunk_size;   /* tokens per chunk for the firing schedule (default 64) */
  int32_t promotion;    /* NGDN2_PROMOTION_* */
  int32_t dtype;        /* element type of o (the reference returns q's dtype) */
  int32_t param_dtype;
  float scale;
  int32_t n_max;
  int32_t n_queries[NGDN2_MAX_LEVELS];
  int32_t firing[NGDN2_MAX_LEVELS];

  const void* q;   int32_t q_dtype;   int64_t q_stride[4];   /* [B, H, L, K] */
  const void* k;   int32_t k_dtype;   int64_t k_stride[3];   /* [B, H, K] */
  const void* v;   int32_t v_dtype;   int64_t v_stride[3];   /* [B, H, V] */
  const void* g;   int32_t g_dtype;   int64_t g_stride[3];   /* [B, H, K] */
  const void* b;   int32_t b_dtype;   int64_t b_stride[3];   /* [B, H, K] */
  const void* w;   int32_t w_dtype;   int64_t w_stride[3];   /* [B, H, V] */
  const void* mix; int32_t mix_dtype; int64_t mix_stride[3]; /* [B, H, L] */

  const void* query_banks;
  const void* key_projections;
  const void* b_projections;
  const void* w_projections;
  const void* g_projections;

  const int64_t* positions;     /* [B] device positions of this token, or NULL */
  int64_t position;             /* the position of every row when positions is NULL */
  const float* state_in;        /* [B, H, L, K, V] contiguous */
  float* state_out;             /* [B, H, L, K, V] contiguous; may equal state_in */
  void* o;                      /* [B, H, V] contiguous, element type dtype */

  void* workspace;              /* >= ngdn2_step_workspace_size */
  size_t workspace_bytes;
  int32_t* status;
} ngdn2_step_args;

/* Arguments of ngdn2_bwd: the gradients of sum(o * d_o) + sum(final * d_final)
 * with respect to every differentiable input of the forward
 * (ChunkNestedGDN2Function.backward, chunk.py:650-719, whose gradient
 * composition is chunk_nested_gdn2_bwd, chunk.py:368-564). Computed on CUDA
 * cores in fp32 from a re-run of the forward. Gradient outputs are fp32 and
 * contiguous in the shape of their input. */
typedef struct ngdn2_bwd_args {
  int32_t abi_version;
  ngdn2_fwd_args fwd;   /* the forward's arguments; its o, final_state,
                           workspace and path are not used */
  const void* d_o; int32_t d_o_dtype; int64_t d_o_stride[4];  /* [B, T, H, V] */
  const float* d_final;        /* [B, H, L, K, V] contiguous, or NULL for zeros */
  float* dq;                   /* [B, T, H, L, K] */
  float* dk;                   /* [B, T, H, K] */
  float* dv;                   /* [B, T, H, V] */
  float* dg;                   /* [B, T, H, K] */
  float* db;                   /* [B, T, H, K] */
  float* dw;                   /* [B, T, H, V] */
  float* dmix;                 /* [B, T, H, L] */
  float* dquery_banks;         /* [L-1, H, n_max, K], or NULL to skip */
  float* dkey_projections;     /* [L-1, H, K, V], or NULL */
  float* db_projections;       /* [L-1, H, V, K], or NULL */
  float* dw_projections;       /* [L-1, H, V, V], or NULL */
  float* dg_projections;       /* [L-1, H, V, K], or NULL */
  float* dinitial_state;       /* [B, H, L, K, V], or NULL */
  void* workspace;             /* >= ngdn2_bwd_workspace_size */
  size_t workspace_bytes;
} ngdn2_bwd_args;

NGDN2_API int ngdn2_abi_version(void);
/* sizeof the argument structs, so bindings can check their layout. */
NGDN2_API size_t ngdn2_sizeof_fwd_args(void);
NGDN2_API size_t ngdn2_sizeof_update_args(void);
NGDN2_API size_t ngdn2_sizeof_step_args(void);
NGDN2_API size_t ngdn2_sizeof_bwd_args(void);
NGDN2_API size_t ngdn2_sizeof_update_bwd_args(void);
NGDN2_API const char* ngdn2_error_string(int code);

/* Validates *args and returns the workspace ngdn2_fwd needs, in bytes. */
NGDN2_API int ngdn2_fwd_workspace_size(const ngdn2_fwd_args* args, size_t* bytes);

/* Which path ngdn2_fwd would run (NGDN2_PATH_SIMT or NGDN2_PATH_TC), or an
 * error code. */
NGDN2_API int ngdn2_fwd_select_path(const ngdn2_fwd_args* args);

/* The forward: o and final_state from the inputs. */
NGDN2_API int ngdn2_fwd(const ngdn2_fwd_args* args, void* stream);

/* One stage of the forward, for profiling: stage 1 launches the
 * chunk-parallel preparation kernels, stage 2 the sequential scan (which
 * reads what stage 1 left in the same workspace); stage 0 is ngdn2_fwd. */
NGDN2_API int ngdn2_fwd_stage(const ngdn2_fwd_args* args, int stage, void* stream);

/* Number of kernel launches ngdn2_fwd makes for these arguments. */
NGDN2_API int ngdn2_fwd_num_launches(const ngdn2_fwd_args* args);

/* Validates *args and returns the workspace ngdn2_bwd needs, in bytes
 * (the forward's records and checkpoints, the per-chunk state gradients and
 * the backward's scratch: about (3 NT + 1) K V + 4 NT 64 (K + V) floats per
 * (batch row, head)). */
NGDN2_API int ngdn2_bwd_workspace_size(const ngdn2_bwd_args* args, size_t* bytes);

/* The backward. Replaces chunk.py:650-719 (ChunkNestedGDN2Function.backward). */
NGDN2_API int ngdn2_bwd(const ngdn2_bwd_args* args, void* stream);

/* Number of kernel launches ngdn2_bwd makes (copies excluded). */
NGDN2_API int ngdn2_bwd_num_launches(const ngdn2_bwd_args* args);

/* The promotion write scan on its own. */
NGDN2_API int ngdn2_update_state(const ngdn2_update_args* args, void* stream);

/* Its backward (update_bwd.py:167-263); same validation and error codes as
 * the forward (update_bwd.py:197-206). */
NGDN2_API int ngdn2_update_bwd_workspace_size(const ngdn2_update_bwd_args* args, size_t* bytes);
NGDN2_API int ngdn2_update_state_bwd(const ngdn2_update_bwd_args* args, void* stream);

/* Validates *args and returns the workspace ngdn2_step needs, in bytes
 * (fp32 parameter copies and promotion scratch). */
NGDN2_API int ngdn2_step_workspace_size(const ngdn2_step_args* args, size_t* bytes);

/* One decode token (naive.py:42-134): level 0 writes, every level is read
 * and mixed into o, then each level whose firing this token completes
 * promotes, bottom-up, per batch row (rows may sit at different positions).
 * Reads state_in, writes state_out (in place when they are equal). */
NGDN2_API int ngdn2_step(const ngdn2_step_args* args, void* stream);

/* Capacity of the fixed scratch buffer behind ngdn2_fwd_noalloc. */
#define NGDN2_NOALLOC_SCRATCH_BYTES ((size_t)64 << 20)

/* The forward without a caller workspace and without any allocation: for
 * callers that cannot allocate device memory per call (a host process that
 * owns all device memory through its own pool, a serving loop whose memory
 * budget is fixed at start-up). It has no counterpart in the reference.
 * args->workspace and args->workspace_bytes are ignored; scratch comes from
 * one buffer of NGDN2_NOALLOC_SCRATCH_BYTES compiled into the library, held
 * on every GPU that loads it until exit. Calls needing more scratch than
 * that return NGDN2_ERR_WORKSPACE. All calls on a device share the buffer,
 * so calls that overlap on the GPU race; the first call on each device
 * looks the buffer up and should come before any stream capture. The looked-up
 * address is cached for the life of the process: after cudaDeviceReset (or
 * any teardown of the device's primary context) this entry point must not be
 * called again in that process. */
NGDN2_API int ngdn2_fwd_noalloc(const ngdn2_fwd_args* args, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* NGDN2_H_ */
