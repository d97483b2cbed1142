/*
 * turboadam_b200.h -- C ABI of the B200-native TurboAdam optimizer step.
 *
 * Plain pointers and sizes only. Every pointer argument named *_dev is a
 * device pointer owned by the caller (the library never allocates or frees
 * device memory); `stream` is a cudaStream_t passed as void*. All compute
 * entry points are asynchronous on that stream; the returned ta_status only
 * reports host-side validation and launch errors. Device-side anomalies
 * (non-finite gradients, a bounded wait that ran out) are OR-ed into a
 * status word in the caller's workspace, read back with ta_read_status().
 *
 * Reference interfaces (davidkny22/turboadam, src/turboadam/...) that each
 * entry point replaces are cited beside it.
 */
#ifndef TURBOADAM_B200_H
#define TURBOADAM_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define TA_API __attribute__((visibility("default")))
#else
#define TA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define TA_ABI_VERSION 4

typedef enum ta_status {
  TA_OK = 0,
  TA_ERR_INVALID = 1,     /* bad argument (null pointer, size, enum)        */
  TA_ERR_ALIGN = 2,       /* a pointer is not 16-byte aligned               */
  TA_ERR_UNSUPPORTED = 3, /* valid in the reference but not built here      */
  TA_ERR_WORKSPACE = 4,   /* workspace too small                            */
  TA_ERR_CUDA = 5         /* a CUDA runtime call failed (see ta_last_error) */
} ta_status;

/* element types of params / grads */
enum { TA_F32 = 0, TA_BF16 = 1 };

/* ta_tensor.flags */
enum {
  TA_M_COSTATE = 1u << 0,   /* first moment is CoState (else fp32 exp_avg)        */
  TA_V_ONEQ = 1u << 1,      /* second moment is 1Q (else fp32 exp_avg_sq)         */
  TA_M_HAS_STATE = 1u << 2, /* CoState holds a previous encoding (not first step) */
  TA_NO_PARAM = 1u << 3,    /* skip weight decay and the parameter update         */
  TA_M_SPANNING = 1u << 4,  /* CoState shard of a tensor split over ranks:
                               alpha and thresholds reduced via ta_step_phase     */
  TA_M_EF = 1u << 6,        /* CoState error feedback (costate.py:410-437): m's
                               EMA takes g + m_ef_dev, and after the encode the
                               residual becomes the EMA of what it lost       */
  TA_M_EF_STATE = 1u << 7,  /* m_ef_dev holds a residual (the reference's
                               _ef_residual is not None)                       */
  TA_EXACT_PARAM = 1u << 5  /* parameter update with correctly rounded v / bc2,
                               sqrt and division: bit-identical to the
                               reference's op sequence (optimizer.py:163-170).
                               Without it they use the hardware estimates
                               (rsqrt, and rcp with one correction of the
                               quotient): the update is within about 3e-7
                               relative of the reference's; no state depends
                               on it, so every packed state bit is the same
                               either way                                      */
};

/* ta_step_phase phases (in call order; the caller all-reduces (sum) the
 * exchange regions between them, see ta_exchange_size) */
enum {
  TA_PHASE_PASS1 = 0,  /* pass 1; spanning alpha chunk sums -> exchange chunks */
  TA_PHASE_PASS2 = 1,  /* alpha from summed chunks, pass 2, histogram round 0 */
  TA_PHASE_SEL1 = 2,   /* pick round 0, histogram round 1                      */
  TA_PHASE_SEL2 = 3,   /* pick round 1, histogram round 2                      */
  TA_PHASE_LABELS = 4  /* pick round 2, labels, commit alpha                    */
};

/* device status bits (ta_read_status) */
enum {
  TA_STATUS_NONFINITE_GRAD = 1u << 0,
  TA_STATUS_WAIT_TIMEOUT = 1u << 1,
  TA_STATUS_BIAS_TABLE_SHORT = 1u << 2  /* ta_step_prepared ran past its bias table */
};

/*
 * One parameter tensor of an optimizer step.
 * Replaces the per-parameter `state` dict of TurboAdam (optimizer.py:242-286)
 * with the same packed layout:
 *   v_idx   compressed_v["indices"]  u8 [B*block]   (quantize.py:134)
 *   v_hdr   compressed_v["scales"]   fp16 [B][2] = (log_min, log_max) of ln v
 *   m_*     CoStateManager._encoded  labels u8[B], sign_packed u8[ceil(n/8)]
 *           (MSB first), block_norms fp32[B], scales fp16[B]; _alpha fp32[1]
 *   exp_avg / exp_avg_sq             fp32 [n]
 * with B = ceil(n / block). State arrays (everything but param/grad) must be
 * allocated with room for a whole number of 16-block tiles:
 * ta_state_padded_blocks(n) blocks (idx: that many * block bytes).
 */
typedef struct ta_tensor {
  void* param_dev;            /* [n] fp32 or bf16, updated in place                */
  const void* grad_dev;       /* [n] same dtype as param                           */
  int64_t numel;              /* n                                                 */
  int32_t dtype;              /* TA_F32 | TA_BF16                                  */
  int32_t group;              /* index into the ta_group array                     */
  uint32_t flags;             /* TA_M_COSTATE | TA_V_ONEQ | ...                    */
  uint32_t tensor_id;         /* stable id of the tensor (stochastic-rounding key) */
  uint32_t step;              /* this tensor's step count after increment (>= 1)   */
  int32_t reserved0;
  uint8_t* v_idx_dev;         /* TA_V_ONEQ                                         */
  uint16_t* v_hdr_dev;        /* TA_V_ONEQ                                         */
  float* exp_avg_sq_dev;      /* !TA_V_ONEQ                                        */
  uint8_t* m_labels_dev;      /* TA_M_COSTATE                                      */
  uint8_t* m_signs_dev;       /* TA_M_COSTATE                                      */
  float* m_norms_dev;         /* TA_M_COSTATE                                      */
  uint16_t* m_amp_dev;        /* TA_M_COSTATE                                      */
  float* m_alpha_dev;         /* TA_M_COSTATE, [1]                                 */
  float* exp_avg_dev;         /* !TA_M_COSTATE                                     */
  const float* sr_uniforms_dev; /* optional [B*block]: replaces the Philox draws   */
  const float* alpha_inject_dev;/* optional [1]: replaces the computed alpha       */
  float* m_out_dev;           /* optional [n]: receives m_new (CoState.update seam)*/
  float* v_out_dev;           /* optional [n]: receives fp32 v_new                 */
  /* shards of a tensor split over ranks (ZeRO-1); 0 for a whole tensor */
  int64_t block_offset;       /* global block index of this shard's block 0; a
                                 multiple of TA_SHARD_ALIGN_BLOCKS when spanning    */
  int64_t global_blocks;      /* blocks of the whole tensor (0: this tensor's)     */
  int64_t exch_chunk_off;     /* TA_M_SPANNING: this tensor's slot in the exchange */
  int64_t exch_hist_off;      /*   regions (ta_exchange_layout), in elements       */
  float* m_ef_dev;            /* TA_M_EF: [n] fp32 error-feedback residual, read
                                 (with TA_M_EF_STATE) and rewritten by the step  */
} ta_tensor;

/* shard boundaries of a spanning tensor fall on multiples of this many blocks
 * (one alpha reduction chunk), which keeps alpha's summation order -- and so
 * every packed bit -- independent of the number of ranks */
#define TA_SHARD_ALIGN_BLOCKS 4096

/*
 * Hyper-parameters of one param group (optimizer.py:67-80 defaults).
 * bc1/bc2 are the fp32 bias corrections 1-beta^t the reference fills into
 * its shared `_bc1/_bc2` tensors (optimizer.py:172-188).
 */
typedef struct ta_group {
  double lr, beta1, beta2, eps, weight_decay;
  double null_pct, amp_pct;
  float bc1, bc2;
  int32_t block_size;         /* only 128 is built                                 */
  int32_t v_bits;             /* 2, 3, 4, 6 or 8                                   */
} ta_group;

/* Library ABI version (TA_ABI_VERSION). */
TA_API int ta_abi_version(void);

/* Message of the last failed call on this thread ("" if none). */
TA_API const char* ta_last_error(void);

/* Blocks to allocate per state array for a tensor of n elements (B rounded up
 * to whole 16-block tiles). */
TA_API int64_t ta_state_padded_blocks(int64_t n, int32_t block_size);

/* Workspace bytes ta_step needs for this tensor list. */
TA_API size_t ta_workspace_size(const ta_tensor* tensors, int32_t n_tensors);

/*
 * One fused optimizer step over a list of tensors.
 * Replaces TurboAdam._full_step_kernel (optimizer.py:88-170), i.e. per tensor
 * decoupled weight decay, the m update (CoStateManager.update,
 * costate.py:367-464, or the fp32 EMA), the v update (fused_v_update,
 * quantize.py:222-299, or the fp32 EMA) and p.addcdiv_ -- as a fixed
 * sequence of multi-tensor kernels (pass 1 over p/g/state, per-tensor alpha,
 * pass 2 CoState encode, exact P10/P90 radix select, labels).
 * seed: 64-bit key of the stochastic-rounding generator.
 */
TA_API ta_status ta_step(const ta_tensor* tensors, int32_t n_tensors, const ta_group* groups,
                  int32_t n_groups, uint64_t seed, void* workspace_dev,
                  size_t workspace_bytes, void* stream);

/*
 * ta_step with timing marks: phase_events[0..4] (cudaEvent_t as void*, any
 * may be NULL) are recorded on `stream` before pass 1, after pass 1, after
 * the alpha reduction, after pass 2 and after the labels kernel, so a caller
 * can time each kernel inside its own timed region. No counterpart in the
 * reference (which has no per-kernel timing); same semantics as ta_step.
 */
TA_API ta_status ta_step_profiled(const ta_tensor* tensors, int32_t n_tensors,
                                  const ta_group* groups, int32_t n_groups, uint64_t seed,
                                  void* workspace_dev, size_t workspace_bytes, void* stream,
                                  void* const* phase_events);

/*
 * Device-resident per-step values of a CUDA-graph-capturable step
 * (ta_step_prepared), so that a graph replay needs nothing from the host.
 */
typedef struct ta_dynamic {
  int32_t* steps_dev;           /* [n_tensors] step counts; each step adds 1     */
  const float* bias_table_dev;  /* [n_groups][table_steps][2] fp32 (1 - beta1^t,
                                   1 - beta2^t) for t = 1..table_steps, computed
                                   on the host exactly as optimizer.py:172-188  */
  int64_t table_steps;
  const double* lr_dev;         /* optional [n_groups] learning rates (else ta_group.lr) */
  const float* grad_scale_dev;  /* optional [1]: AMP loss scale; gradients enter
                                   the step multiplied by RN(1 / scale), as
                                   GradScaler.unscale_ leaves them           */
  const float* found_inf_dev;   /* optional [1]: nonzero skips the whole step
                                   (step counts included)                    */
} ta_dynamic;

/*
 * Uploads the descriptor table of a tensor list into the workspace (one
 * stream-ordered host-to-device copy). Call it outside any stream capture,
 * again whenever a pointer, size or group setting changes.
 * No counterpart in the reference (capturable=True raises there).
 */
TA_API ta_status ta_plan_prepare(const ta_tensor* tensors, int32_t n_tensors,
                                 const ta_group* groups, int32_t n_groups, uint64_t seed,
                                 void* workspace_dev, size_t workspace_bytes, void* stream);

/*
 * ta_step on a prepared workspace with its per-step values taken from device
 * memory: one small kernel advances the step counts, bias corrections, flags
 * and (optional) learning rates and loss scale, then the step's kernels run.
 * Only kernel launches: it can be captured into a CUDA graph and replayed.
 * The step / TA_M_HAS_STATE fields of `tensors` are ignored (device counts).
 * No counterpart in the reference.
 */
TA_API ta_status ta_step_prepared(const ta_tensor* tensors, int32_t n_tensors,
                                  const ta_group* groups, int32_t n_groups, uint64_t seed,
                                  void* workspace_dev, size_t workspace_bytes,
                                  const ta_dynamic* dyn, void* stream);

/*
 * Layout of the exchange buffer of a sharded step, the same on every rank:
 * for the n tensors split over ranks (the whole job's list, in one agreed
 * order; global_blocks[i] blocks each) it returns each tensor's slot --
 * chunk_off[i] in fp64 elements of the chunk region ([2][alpha chunks] per
 * tensor), hist_off[i] in uint32 elements of the histogram region ([2][2048]
 * per tensor) -- and the two region sizes (the histogram region follows the
 * chunk region in the buffer). Copy the slots into exch_chunk_off /
 * exch_hist_off of the rank's shards. No counterpart in the reference
 * (single-process); the reductions it carries are costate.py:22-43, :94-118.
 */
TA_API ta_status ta_exchange_layout(const int64_t* global_blocks, int32_t n, int64_t* chunk_off,
                                    int64_t* hist_off, size_t* chunk_bytes,
                                    size_t* hist_bytes);

/*
 * One phase of a sharded optimizer step (ZeRO-1). Every rank calls the five
 * phases in order on the same layout; between them the caller all-reduces
 * (sums over ranks) the chunk region after TA_PHASE_PASS1 and the histogram
 * region after PASS2, SEL1 and SEL2 -- on every rank, also on ranks that hold
 * no split tensor. Each rank then holds exactly the packed state the
 * unsharded ta_step gives its shards. Tensors without TA_M_SPANNING complete
 * as in ta_step. TA_PHASE_PASS1 uploads the step's descriptor table into the
 * workspace and the later phases run on it: pass the same tensor and group
 * arrays to all five calls of a step. No counterpart in the reference.
 */
TA_API ta_status ta_step_phase(const ta_tensor* tensors, int32_t n_tensors,
                               const ta_group* groups, int32_t n_groups, uint64_t seed,
                               void* workspace_dev, size_t workspace_bytes, void* exchange_dev,
                               size_t chunk_bytes, size_t hist_bytes, int32_t phase,
                               void* stream);

/* Reads (and optionally clears) the device status word of a workspace
 * (synchronises the stream). */
TA_API ta_status ta_read_status(void* workspace_dev, int32_t clear, uint32_t* status_out,
                         void* stream);

/*
 * 1Q fused v update of one tensor.
 * Replaces quantize.fused_v_update (quantize.py:222-299) and
 * triton_kernels.triton_fused_v_update (triton_kernels.py:105-165).
 * idx/hdr are read, out_idx/out_hdr written (may alias the inputs).
 * uniforms_dev: optional [B*block] draws (else Philox keyed by seed,
 * tensor_id, step). v_out_dev: [n] fp32 v_new.
 */
TA_API ta_status ta_v_update(const uint8_t* idx_dev, const uint16_t* hdr_dev, const void* grad_dev,
                      int32_t grad_dtype, int64_t n, int32_t block_size, int32_t v_bits,
                      double beta2, const float* uniforms_dev, uint64_t seed,
                      uint32_t tensor_id, uint32_t step, uint8_t* out_idx_dev,
                      uint16_t* out_hdr_dev, float* v_out_dev, void* workspace_dev,
                      size_t workspace_bytes, void* stream);

/*
 * ta_v_update without a caller workspace. No counterpart in the reference:
 * the scratch that ta_v_update carves from workspace_dev lives in a
 * file-scope static device array of TA_V_UPDATE_NOALLOC_SCRATCH_BYTES per
 * device, so the call allocates no device memory. n above
 * TA_V_UPDATE_NOALLOC_MAX_N is rejected with TA_ERR_UNSUPPORTED.
 * Every call looks up the array's device address on the current device (no
 * allocation); the first call on a device, and the first after a context
 * reset reloaded the module, zeroes the whole array on `stream` -- make that
 * call before any stream capture. Each call then clears the array's status
 * word (its first 4 bytes) and the kernels OR into it what the workspace
 * entry points report through ta_read_status (TA_STATUS_NONFINITE_GRAD,
 * TA_STATUS_WAIT_TIMEOUT); ta_v_update_noalloc_status reads it. Every other
 * scratch byte is written by the call before it is read.
 * All calls on one device share the array: calls that can overlap (other
 * streams, other host threads, without ordering) race; serialise them.
 * Arguments and results as ta_v_update.
 */
#define TA_V_UPDATE_NOALLOC_MAX_N ((int64_t)1 << 20)
#define TA_V_UPDATE_NOALLOC_SCRATCH_BYTES ((size_t)5 << 18) /* 1.25 MiB */
TA_API ta_status ta_v_update_noalloc(const uint8_t* idx_dev, const uint16_t* hdr_dev,
                                     const void* grad_dev, int32_t grad_dtype, int64_t n,
                                     int32_t block_size, int32_t v_bits, double beta2,
                                     const float* uniforms_dev, uint64_t seed,
                                     uint32_t tensor_id, uint32_t step, uint8_t* out_idx_dev,
                                     uint16_t* out_hdr_dev, float* v_out_dev, void* stream);

/*
 * Device status of the last ta_v_update_noalloc call on the current device
 * (TA_STATUS_* bits), read from the static array's status word after
 * `stream` is synchronised; clear != 0 zeroes the word afterwards. No
 * counterpart in the reference; ta_read_status's counterpart for the entry
 * point that has no caller workspace.
 */
TA_API ta_status ta_v_update_noalloc_status(int32_t clear, uint32_t* status_out, void* stream);

/* 1Q state of a fresh tensor: compress_v_logscale(full(1e-30)) as done at
 * optimizer.py:273-280 (all indices 0, both headers fp16(ln 1e-30)). */
TA_API ta_status ta_v_init(int64_t n, int32_t block_size, uint8_t* idx_dev, uint16_t* hdr_dev,
                    void* stream);

/* Decode 1Q state to fp32 v.
 * Replaces oneq.decompress_v (oneq.py:51-67) / quantize.dequantize_logscale_nbits
 * (quantize.py:183-214). */
TA_API ta_status ta_v_decode(const uint8_t* idx_dev, const uint16_t* hdr_dev, int64_t n,
                      int32_t block_size, int32_t v_bits, float* v_out_dev, void* stream);

/* CoState decode m_hat = alpha*g + scale*sign.
 * Replaces costate.decode_blocks (costate.py:261-323) and
 * triton_kernels.triton_costate_decode (triton_kernels.py:217-261). */
TA_API ta_status ta_costate_decode(const uint8_t* labels_dev, const uint8_t* signs_dev,
                            const float* norms_dev, const uint16_t* amp_dev,
                            const float* alpha_dev, const void* grad_dev,
                            int32_t grad_dtype, int64_t n, int32_t block_size,
                            float* m_out_dev, void* stream);

/* CoState encode (block norms, fp16 amplitude scales, MSB-first sign bits).
 * Replaces costate.encode_blocks (costate.py:213-258) and
 * triton_kernels.triton_costate_encode (triton_kernels.py:313-358). */
TA_API ta_status ta_costate_encode(const float* delta_dev, int64_t n, int32_t block_size,
                            uint8_t* signs_dev, float* norms_dev, uint16_t* amp_dev,
                            void* stream);

/* Exact P-quantile thresholds of per-block ratios (fp32-bit radix select).
 * Replaces costate.compute_thresholds (costate.py:94-118); tau_dev[0..1] =
 * (tau0, tau1). Also writes labels (costate.classify_blocks,
 * costate.py:126-149) when labels_dev is not NULL. */
TA_API ta_status ta_thresholds(const float* ratios_dev, int64_t n_blocks, double null_pct,
                        double amp_pct, float* tau_dev, uint8_t* labels_dev,
                        void* workspace_dev, size_t workspace_bytes, void* stream);

/* Workspace bytes for ta_v_update / ta_thresholds on n elements / blocks. */
TA_API size_t ta_aux_workspace_size(int64_t n);

/*
 * Device self-test of the hardware-estimate properties the step relies on.
 * No counterpart in the reference (its arithmetic is torch's CPU ops).
 * Over every normal binary32 x it writes
 *   out_dev[0] = bits of the double max |RN(ln2 * lg2.approx(x)) - ta_logf(x)|
 *                over x with ta_logf(x) >= -69.3 (the certified
 *                re-quantisation assumes <= 2^-16),
 *   out_dev[1] = number of adjacent normal pairs x < x' with
 *                ta_logf(x') < ta_logf(x) (the step assumes 0),
 *   out_dev[2] = number of x with a normal 1/x where rcp.approx plus one
 *                Newton step differs from RN(1/x) (the fast reciprocals of
 *                the step assume 0),
 *   out_dev[3] = bits of the double max relative error of rsqrt.approx(x),
 *   out_dev[4] = bits of the double max relative error of rcp.approx(x) over
 *                x with a normal 1/x (the default parameter update assumes
 *                both <= 2^-22),
 *   out_dev[5] = number of non-NaN binary32 x (either sign, zeros,
 *                subnormals and infinities included) whose hardware
 *                bfloat16 rounding (cvt.rn.bf16x2.f32, used by the bf16
 *                parameter stores) differs from the portable
 *                round-to-nearest-even (the step assumes 0).
 * out_dev: 6 uint64 in device memory, zeroed by the caller.
 */
TA_API ta_status ta_selftest_fast_math(uint64_t* out_dev, void* stream);

/*
 * Device self-test of the bounded waits of the step's pipelines. No
 * counterpart in the reference. One CTA shaped like the pass kernels arms a
 * stage for a copy that never lands (none is issued): its consumer warps'
 * waits run out after limit_ns (0 < limit_ns <= 2e9; the step uses 2 s) and
 * they skip the stage, the producer's wait for them runs out too, and every
 * thread returns. It ORs TA_STATUS_WAIT_TIMEOUT into *status_dev and writes
 * out_dev[0] = the CTA's elapsed nanoseconds (%globaltimer), out_dev[1] =
 * the number of waits that ran out (5). The context stays usable.
 */
TA_API ta_status ta_selftest_wait_timeout(uint64_t limit_ns, uint32_t* status_dev,
                                          uint64_t* out_dev, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TURBOADAM_B200_H */
