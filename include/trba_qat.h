/*
 * trba_qat.h — the fused, device-resident INT8-QAT training step of
 * libtrba_b200.so (new entry points; no counterpart in the reference's C ABI).
 *
 * One call runs what the reference's return_main_step (later snapshot
 * src/main.rs:2249-2413) runs across its Rust host and backend: SE-ResNet
 * QAT forward/backward (src/qnet.rs), 2-layer BiLSTM (src/rnn.rs), attention
 * decoder (src/attn.rs), CE + CTC losses (src/main.rs:2300-2336,
 * src/ctc.rs), global-norm clip, Muon for matrices and Adam for vectors
 * (src/opt.rs, device conv Muon src/qnet.rs:559-573) and the QAT weight
 * re-quantisation — with every scale, statistic and gradient kept on the
 * device (no host round trip inside the step).
 *
 * Parameters live in one flat fp32 buffer in the reference's manifest order
 * (Model::params_filtered, src/main.rs:954-1030); gradients in a second
 * buffer of the same layout, which is what data-parallel training
 * all-reduces.  All pointers passed to *_dev functions are device pointers;
 * *_host functions take host pointers (pinned for asynchronous copies).
 * Functions return 0 on success, a negative value on invalid arguments and a
 * positive CUDA error code otherwise.
 */
#ifndef TRBA_QAT_H
#define TRBA_QAT_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct trba_model trba_model;

typedef struct {
    int fd;           /* feature width (src/qnet.rs:1430: widths fd/8 .. fd)   */
    int hidden;       /* BiLSTM / decoder hidden size                           */
    int classes;      /* vocabulary incl. pad 0, sos 1, eos 2                   */
    int img_h, img_w; /* input image (int8, NCHW, scale 1/127)                  */
    int max_len;      /* decoder steps = max_len + 1                            */
    int rnn_layers;
    int batch;        /* largest batch a step may use (buffers are sized once)  */
    int sos, eos, pad;
    float lr, weight_decay, ctc_weight, muon_cap;
    int clip_warmup;  /* steps with global-norm clipping at 5.0                 */
    int wgrad_mode;   /* 0: reference-compatible operand order, 1: dW = dX^T col */
    int dgrad_mode;   /* conv input gradient: 0 exact (the reference's f32 order, CUDA cores),
                         1 tensor cores (implicit GEMM, fp32 dy as three bf16 terms) */
    int wq_per_channel; /* conv weight quantisation: 0 per tensor (the reference, src/qnet.rs:316-331),
                           1 per output channel (scale max |w[row]| / 127 for each row) */
    int inference_only; /* 1: allocate the forward path only (no gradients, optimiser state or
                           backward traces); training entry points then return -3 */
    int conv_fwd_mode;  /* conv forward GEMM: 0 im2col matrix + GEMM (the reference's two launches),
                           1 (default) implicit GEMM for Cin a power of two >= 16: the operand is
                           gathered from the activations, and in training the weight gradient's
                           im2col operand is built off the forward path, beside the sequence
                           head.  Same s32 accumulators either way. */
} trba_model_config;

/* TRBA-small defaults (fd 128, hidden 64, 130 classes, 32x160, max_len 20). */
void trba_model_default_config(trba_model_config *cfg);

trba_model *trba_model_create(const trba_model_config *cfg);
void trba_model_destroy(trba_model *m);

/* Parameter manifest: count of entries and of floats; entry i gives its name,
 * offset (floats) in the flat buffer, matrix shape (cols = 0 for vectors) and
 * kind (0 conv weight: device Muon, 1 matrix: Muon, 2 vector: Adam). */
long long trba_model_param_count(const trba_model *m);
int trba_model_param_entries(const trba_model *m);
int trba_model_param_entry(const trba_model *m, int i, char *name, int name_cap, long long *offset, int *rows,
                           int *cols, int *kind);

/* Copy the whole parameter vector in / out (host fp32, manifest order).
 * set_params also re-quantises the conv weights and resets optimiser state. */
int trba_model_set_params(trba_model *m, const float *host, long long n);
int trba_model_get_params(trba_model *m, float *host, long long n);
/* Gradients of the last forward_backward (before clipping / averaging). */
int trba_model_get_grads(trba_model *m, float *host, long long n);
float *trba_model_grad_buffer(trba_model *m);

/* Forward + backward on device inputs: img [B,3,H,W] int8; text_in, target
 * [B, max_len+1] int32; ctc_tgt [B, max_len+1] int32 with lengths ctc_len
 * [B] (tokens plus eos).  Leaves the loss in trba_model_loss_dev(). */
int trba_model_forward_backward(trba_model *m, const int8_t *img, const int32_t *text_in, const int32_t *target,
                                const int32_t *ctc_tgt, const int32_t *ctc_len, int batch, void *stream);
/* Inference (run_inference, later snapshot src/main.rs:2690; greedy
 * decoding src/attn.rs:368-447): the CNN with BN running statistics, the
 * BiLSTM stack, greedy attention decoding from sos.  step_tokens (device,
 * [max_len+1, batch] int32, or NULL for the model's own buffer) receives the
 * argmax token of every decoding step. */
int trba_model_infer(trba_model *m, const int8_t *img, int batch, int32_t *step_tokens, void *stream);
/* The same from a host image batch, with the reference's output rule: eos is
 * not emitted and decoding stops after the first step at which every sample
 * produced eos.  tokens (host, [batch, max_len+1]) gets each sample's tokens
 * followed by -1, lengths (host, [batch]) their counts.  Synchronises. */
int trba_model_infer_host(trba_model *m, const int8_t *img, int batch, int32_t *tokens, int32_t *lengths,
                          void *stream);
/* Clip (first clip_warmup steps), Muon/Adam, re-quantise. */
int trba_model_optimizer_step(trba_model *m, void *stream);
/* forward_backward, gradient all-reduce (when data-parallel), optimizer_step. */
int trba_model_train_step(trba_model *m, const int8_t *img, const int32_t *text_in, const int32_t *target,
                          const int32_t *ctc_tgt, const int32_t *ctc_len, int batch, void *stream);
/* The same step from host buffers: copies the inputs in, runs the step and
 * copies the three losses (total, attention CE, CTC) back into loss_host. */
int trba_model_train_step_host(trba_model *m, const int8_t *img, const int32_t *text_in, const int32_t *target,
                               const int32_t *ctc_tgt, const int32_t *ctc_len, int batch, float *loss_host,
                               void *stream);
/* Device pointer to 4 floats: total loss, attention CE, CTC, CE grad scale. */
const float *trba_model_loss_dev(const trba_model *m);
/* Device pointer to the model's [max_len+1, batch] greedy-decoding tokens. */
const int32_t *trba_model_step_tokens_dev(const trba_model *m);
/* Batch-norm running statistics (mean then var, conv manifest order). */
int trba_model_get_running_stats(trba_model *m, float *host, long long n);
long long trba_model_running_stats_count(const trba_model *m);
/* Number of optimizer steps taken. */
long long trba_model_step_count(const trba_model *m);
/* Bytes of device memory the model holds. */
long long trba_model_device_bytes(const trba_model *m);

/* Optimiser state and BN running statistics in and out, for checkpoints
 * (src/main.rs:1099-1193 of the later snapshot saves them): the Adam first /
 * second moments of every parameter (manifest order, zero where Adam is not
 * used), the running statistics in trba_model_get_running_stats' order, and
 * the optimiser step count.  set_params resets all three, so restore them
 * after it. */
int trba_model_get_moments(trba_model *m, float *m_host, float *v_host, long long n);
int trba_model_set_moments(trba_model *m, const float *m_host, const float *v_host, long long n);
int trba_model_set_running_stats(trba_model *m, const float *host, long long n);
int trba_model_set_step_count(trba_model *m, long long t);

/* Diagnostics: copy an internal fp32 buffer of the last step to the host
 * (feat, dfeat, enc, d_enc, logits, dlogits, ctc_logits, dctc, <conv>.x,
 * <conv>.mean, <conv>.var); n must equal the buffer's element count. */
int trba_model_debug_tensor(trba_model *m, const char *name, float *host, long long n);

/* Kernel probe (no counterpart in the reference): while a kind is set, every
 * launch of that kernel family in the step is bracketed by CUDA events on the
 * step's stream, and its algorithmic work is summed: arithmetic operations
 * (2*M*N*K for the GEMMs; one multiply and one add per gather term for the
 * input gradient) and bytes (one read of every input, one write of every
 * output).  trba_model_probe(m, kind) selects a kind (-1 = off) and clears
 * the record; trba_model_probe_read waits for the last event and returns the
 * summed device milliseconds, launches, operations and bytes. */
#define TRBA_PROBE_CONV_GEMM 0  /* conv forward int8 tcgen05 GEMM (+BN sums epilogue) */
#define TRBA_PROBE_WGRAD_GEMM 1 /* conv weight-gradient int8 tcgen05 split-K GEMM */
#define TRBA_PROBE_DGRAD 2      /* conv input-gradient gather (fp32, reference summation order) */
#define TRBA_PROBE_SGEMM 3      /* sequence-head fp32 GEMMs (f64 accumulation) */
/* Whole phases of the step on the step's stream (one span per step each):
 * SE-ResNet forward, sequence head forward with the losses, sequence head
 * backward, SE-ResNet backward (until the input-gradient side stream has
 * joined), gradient all-reduce + clip + optimiser + re-quantisation. */
#define TRBA_PROBE_PHASE_CNN_FWD 4
#define TRBA_PROBE_PHASE_HEAD_FWD 5
#define TRBA_PROBE_PHASE_HEAD_BWD 6
#define TRBA_PROBE_PHASE_CNN_BWD 7
#define TRBA_PROBE_PHASE_OPTIMIZER 8
int trba_model_probe(trba_model *m, int kind);
int trba_model_probe_read(trba_model *m, double *ms_total, long long *launches, double *ops, double *bytes,
                          long long *steps);

/* CUDA-graph execution of the step (no counterpart in the reference).  With
 * enable != 0, trba_model_train_step records the whole step (forward,
 * backward, gradient all-reduce, optimiser) into a CUDA graph the first time
 * it sees a set of input pointers, batch and probe kind — recording runs
 * nothing — and replays that graph on later calls with the same pointers:
 * callers refresh the input buffers in place.  Every step-dependent scalar
 * (the optimiser's step count, clip switch and bias corrections) lives on the
 * device, so replays compute exactly what eager steps compute.
 * trba_model_train_step_host stages into the model's own input buffers and so
 * always replays one graph.  A probe selected before the recording is
 * recorded with it: each probed launch is bracketed by two one-thread
 * kernels that write the device's %globaltimer (an event recorded inside a
 * graph cannot be timed), and trba_model_probe_read then reports the
 * launches of the latest replay (steps = 1). */
int trba_model_use_graphs(trba_model *m, int enable);

/* ---- data parallel (one process per GPU, NCCL over NVLink) ---- */
/* 128-byte NCCL unique id from rank 0, broadcast by the caller. */
int trba_dp_unique_id(void *id128);
/* Join the NCCL communicator; afterwards train_step all-reduces (averages)
 * the gradient buffer before the optimizer step. */
int trba_dp_init(trba_model *m, const void *id128, int rank, int world);
int trba_dp_finalize(trba_model *m);
/* Failure detection for data-parallel steps (no counterpart in the
 * reference, which has no multi-GPU path): waits until the work queued on
 * `stream` (a step and its all-reduce) has finished, polling the stream and
 * ncclCommGetAsyncError every 100 us.  An asynchronous NCCL error (a peer
 * that failed) or more than timeout_ms without completion aborts the
 * communicator (ncclCommAbort, which also ends an all-reduce stuck waiting
 * for a peer) and leaves the model single-rank.  Returns 0 when the work
 * finished, 1 after an NCCL error, 2 after a timeout, negative on a CUDA
 * error of the stream. */
int trba_dp_wait(trba_model *m, void *stream, double timeout_ms);
/* The decision loop of trba_dp_wait over caller-supplied probes:
 * stream_done(ctx) returns 1 when the work finished, 0 while pending,
 * negative on error (returned as is); async_error(ctx) returns non-zero for
 * a communicator error; abort_comm(ctx) is called once before returning 1
 * (error) or 2 (timeout_ms passed); poll_us between polls. */
int trba_dp_watch(int (*stream_done)(void *), int (*async_error)(void *), void (*abort_comm)(void *), void *ctx,
                  double timeout_ms, double poll_us);

#ifdef __cplusplus
}
#endif
#endif
