/*
 * cherimoya_b200.h -- C ABI of libcherimoya_b200.so, the sm_100a (B200)
 * inference engine for the Cherimoya model's hot path.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t.
 * None allocates device memory: the caller passes the workspace, sized by
 * the matching *_workspace_bytes() query, so calls can be captured in a
 * CUDA graph. Calls are asynchronous on `stream` and return a chm_status;
 * nothing aborts the process. Device-side waits are bounded; a wait that
 * gives up records CHM_ERR_DEVICE_TIMEOUT in the workspace status word,
 * which chm_read_status() returns after synchronising the stream.
 *
 * Upstream interfaces replaced (paths relative to the upstream project):
 *   chm_forward  -> Cherimoya._forward_impl, CUDA no_grad branch
 *                   (cherimoya/cherimoya.py:340-400), including the per-block
 *                   Triton inference path CheriBlock.forward ->
 *                   _fwd_inf_forward (cherimoya/cheri.py:741-754, 1072-1082)
 *   chm_pack_weights -> CheriBlock eval-time weight cache
 *                   (cherimoya/cheri.py:1004-1025, 1040-1070): bf16 casts with
 *                   residual_scale folded into linear2
 *   chm_ism      -> the saturation-mutagenesis driver the upstream CLI calls
 *                   (cherimoya_cli/commands/attribute.py:54-64), scoring
 *                   delta log-counts and profile Jensen-Shannon distance
 *                   (cherimoya/performance.py:171-207)
 *   chm_variant  -> ref/alt variant-effect scoring
 *                   (docs/tutorials/variant_effect.rst:50-69)
 */
#ifndef CHERIMOYA_B200_H
#define CHERIMOYA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CHM_ABI_VERSION 1

/* Opaque stream handle; identical to cudaStream_t. */
typedef struct CUstream_st* chm_stream_t;

typedef enum {
    CHM_OK = 0,
    CHM_ERR_INVALID_ARGUMENT = 1, /* null pointer, bad size, bad dtype       */
    CHM_ERR_UNSUPPORTED = 2,      /* configuration the kernels do not cover  */
    CHM_ERR_WORKSPACE = 3,        /* workspace / packed buffer too small     */
    CHM_ERR_LAUNCH = 4,           /* a kernel launch failed                  */
    CHM_ERR_DEVICE_TIMEOUT = 5,   /* a bounded device-side wait gave up      */
    CHM_ERR_CUDA = 6              /* another CUDA runtime error              */
} chm_status;

/* Arithmetic of the block stack. Both modes run the MLP contractions as
 * bf16 x bf16 -> fp32 tcgen05 MMAs with fp32 conv/LayerNorm statistics.
 *  CHM_MODE_FP32: fp32 residual stream in HBM, fp32 stem and heads.
 *  CHM_MODE_BF16: bf16 residual stream (the upstream autocast-bf16 mode),
 *                 fp32 stem/head accumulation. */
typedef enum { CHM_MODE_FP32 = 0, CHM_MODE_BF16 = 1 } chm_mode;

/* Input element type of chm_forward's one-hot / dense input. */
typedef enum { CHM_INPUT_F32 = 0, CHM_INPUT_BF16 = 1 } chm_input_dtype;

/* Model hyper-parameters: the constructor arguments of upstream
 * Cherimoya.__init__ (cherimoya/cherimoya.py:148-151) that shape the
 * forward pass, plus the sequence length and the arithmetic mode. */
typedef struct {
    int32_t n_filters;        /* C                                          */
    int32_t n_layers;         /* block i uses dilation 2**i                 */
    int32_t expansion;        /* H = expansion * C                          */
    int32_t n_outputs;        /* sum(signal_groups): profile channels       */
    int32_t n_groups;         /* len(signal_groups): count heads            */
    int32_t n_control_tracks; /* extra profile-head input channels          */
    int32_t trimming;         /* T: profile/count window is [T, L - T)      */
    int32_t seq_len;          /* L                                          */
    float residual_scale;     /* rs (0.15 by default)                       */
    int32_t mode;             /* chm_mode                                   */
} chm_model_desc;

/* Device pointers to the fp32 parameters in the checkpoint's shapes
 * (state_dict layout, cherimoya/cherimoya.py:246-278). The per-layer
 * fields are HOST arrays of n_layers DEVICE pointers. */
typedef struct {
    const float* iconv_weight;            /* (C, 4, 21)                   */
    const float* iconv_bias;              /* (C)                          */
    const float* const* conv_weight;      /* [n_layers] -> (3, C)         */
    const float* const* linear1_weight;   /* [n_layers] -> (H, C)         */
    const float* const* linear2_weight;   /* [n_layers] -> (C, H)         */
    const float* fconv_weight;            /* (n_outputs, C + n_ctl, 75)   */
    const float* fconv_bias;              /* (n_outputs)                  */
    const float* linear_weight;           /* (n_groups, C + (n_ctl > 0))  */
    const float* linear_bias;             /* (n_groups)                   */
} chm_params;

/* Library / ABI introspection. */
int32_t chm_abi_version(void);
const char* chm_error_string(int32_t status);

/* Checks the configuration against what the kernels cover. */
int32_t chm_validate(const chm_model_desc* desc);

/* Bytes of the packed (device-resident, kernel-layout) weight buffer. */
size_t chm_packed_weights_bytes(const chm_model_desc* desc);

/* Packs fp32 parameters into `packed` (device, 1024-byte aligned):
 * bf16 tcgen05 operand tiles in the 128-byte-swizzled K-major layout, with
 * residual_scale folded into linear2 (upstream cheri.py:1021-1024). */
int32_t chm_pack_weights(const chm_model_desc* desc, const chm_params* params,
                         void* packed, size_t packed_bytes, chm_stream_t stream);

/* Workspace bytes chm_forward needs for `batch` sequences. */
size_t chm_forward_workspace_bytes(const chm_model_desc* desc, int32_t batch);

/* Full forward: x (batch, 4, L) one-hot or dense (input_dtype), x_ctl
 * (batch, n_control_tracks, L) fp32 or NULL. Writes profile
 * (batch, n_outputs, L - 2T) fp32 and logcounts (batch, n_groups) fp32.
 * Upstream: Cherimoya._forward_impl (cherimoya/cherimoya.py:340-400). */
int32_t chm_forward(const chm_model_desc* desc, const void* packed, int32_t batch,
                    const void* x, int32_t input_dtype, const float* x_ctl,
                    float* profile, float* logcounts,
                    void* workspace, size_t workspace_bytes, chm_stream_t stream);

/* Same forward with the input given as base indices: bases (batch, L) int8
 * in 0..3 (A, C, G, T); any other value is an all-zero column (N base). */
int32_t chm_forward_bases(const chm_model_desc* desc, const void* packed, int32_t batch,
                          const int8_t* bases, const float* x_ctl,
                          float* profile, float* logcounts,
                          void* workspace, size_t workspace_bytes, chm_stream_t stream);

/* Workspace bytes chm_ism needs when it scores up to `mutant_batch`
 * mutants per pass (the pass size bounds memory, not the problem size). */
size_t chm_ism_workspace_bytes(const chm_model_desc* desc, int32_t n_seqs,
                               int32_t mutant_batch);

/* Saturation mutagenesis of positions [start, end) of each of n_seqs
 * reference sequences (bases, (n_seqs, L) int8). For sequence n, base b and
 * position p the mutant carries b at p; outputs (n_seqs, 4, end - start):
 *   d_logcount = logcount_0(mutant) - logcount_0(reference)
 *   jsd        = Jensen-Shannon distance between softmax(profile(reference))
 *                and softmax(profile(mutant)), flattened over channels and
 *                positions (upstream performance.py:171-207 semantics).
 * Entries with b equal to the reference base are exactly 0. */
int32_t chm_ism(const chm_model_desc* desc, const void* packed, int32_t n_seqs,
                const int8_t* bases, int32_t start, int32_t end, int32_t mutant_batch,
                float* d_logcount, float* jsd,
                void* workspace, size_t workspace_bytes, chm_stream_t stream);

/* chm_ism plus, when d_profile_wrapper is not null, the change of the
 * ProfileWrapper value (upstream cherimoya/wrappers.py:71-99: the flattened
 * profile logits, mean-centred, weighted by their softmax and summed) in
 * every mutant, (n_seqs, 4, end - start), 0 at the reference base. With
 * d_logcount (group g) this is the scalar each upstream attribution target
 * (LogCountWrapper / ProfileWrapper over ControlWrapper, the two outputs of
 * cherimoya_cli/commands/attribute.py:46-51) takes in the mutant minus in the
 * reference. Same workspace as chm_ism. */
int32_t chm_ism_ex(const chm_model_desc* desc, const void* packed, int32_t n_seqs,
                   const int8_t* bases, int32_t start, int32_t end, int32_t mutant_batch,
                   float* d_logcount, float* jsd, float* d_profile_wrapper,
                   void* workspace, size_t workspace_bytes, chm_stream_t stream);

/* Output-wrapper epilogues on a forward's outputs (profile (batch, n_outputs,
 * L - 2T) and logcounts (batch, n_groups), fp32, device):
 *   expected_counts (same shape as profile; skipped when null): per signal group
 *     (group_sizes: n_groups host ints summing to n_outputs) a joint softmax over
 *     the group's channels and positions times expm1(logcount) -- upstream
 *     ExpectedCountsWrapper, cherimoya/wrappers.py:125-166;
 *   profile_wrapper (batch floats; skipped when null): the flattened logits,
 *     mean-centred, weighted by their softmax and summed -- upstream
 *     ProfileWrapper, cherimoya/wrappers.py:71-99; needs a workspace of
 *     batch * n_outputs * (L - 2T) floats. */
int32_t chm_wrapper_epilogue(const chm_model_desc* desc, int32_t batch, const float* profile,
                             const float* logcounts, const int32_t* group_sizes,
                             float* expected_counts, float* profile_wrapper,
                             void* workspace, size_t workspace_bytes, chm_stream_t stream);

/* Workspace bytes chm_variant needs for n_pairs pairs. */
size_t chm_variant_workspace_bytes(const chm_model_desc* desc, int32_t n_pairs);

/* Ref/alt scoring of n_pairs pairs (ref_bases, alt_bases: (n_pairs, L)
 * int8): d_logcount (n_pairs, n_groups) = logcount(alt) - logcount(ref);
 * jsd (n_pairs) between softmax(profile(ref)) and softmax(profile(alt)). */
int32_t chm_variant(const chm_model_desc* desc, const void* packed, int32_t n_pairs,
                    const int8_t* ref_bases, const int8_t* alt_bases,
                    float* d_logcount, float* jsd,
                    void* workspace, size_t workspace_bytes, chm_stream_t stream);

/* ---- one Cheri Block (standalone CheriBlock.forward, upstream
 * cherimoya/cheri.py:1072-1082 -> _fwd_inf_forward, cheri.py:741-754) ---- */

/* Bytes of one block's packed weights (n_filters C, hidden H = expansion*C). */
size_t chm_block_packed_bytes(int32_t n_filters, int32_t hidden);

/* Packs conv_weight (3, C), linear1.weight (H, C) and linear2.weight (C, H)
 * (fp32, device) with residual_scale folded into linear2. */
int32_t chm_pack_block(int32_t n_filters, int32_t hidden, float residual_scale,
                       const float* conv_weight, const float* linear1_weight,
                       const float* linear2_weight, void* packed, size_t packed_bytes,
                       chm_stream_t stream);

/* Workspace bytes chm_block_forward needs. */
size_t chm_block_workspace_bytes(int32_t batch, int32_t seq_len, int32_t n_filters,
                                 int32_t x_dtype);

/* out = x + rs * W2 gelu(W1 LN(dwconv_dilation(x))) for x (batch, L, C),
 * contiguous, fp32 or bf16 (x_dtype, chm_input_dtype); out has x's shape
 * and type and must not alias x. */
int32_t chm_block_forward(int32_t batch, int32_t seq_len, int32_t n_filters, int32_t hidden,
                          int32_t dilation, int32_t x_dtype, const void* packed, const void* x,
                          void* out, void* workspace, size_t workspace_bytes,
                          chm_stream_t stream);

/* ---- forward without any device allocation ----
 * No counterpart in the upstream project. For callers that cannot allocate
 * device memory: a plugin host that owns every device buffer and lends only
 * inputs and outputs, a foreign-language binding with no access to a device
 * allocator, or code that must not call cudaMalloc (which can synchronise
 * the device). Same computation and arguments as chm_forward minus the
 * workspace: the scratch lives in a static device array of
 * CHM_NOALLOC_SCRATCH_BYTES that every GPU loading the library holds until
 * process exit. A batch whose scratch needs more than that is rejected with
 * CHM_ERR_WORKSPACE (the default model at 2114 bp fits about 30 sequences per
 * call in bf16 mode, 15 in fp32 mode). The first call on a device looks up
 * the array's device address (cudaGetSymbolAddress) with that device
 * current; make that first call before any stream capture. All calls share
 * the one array, so calls that overlap on the GPU (different streams, or
 * different host threads) race: order them. */
#define CHM_NOALLOC_SCRATCH_BYTES (32u << 20)
int32_t chm_forward_noalloc(const chm_model_desc* desc, const void* packed, int32_t batch,
                            const void* x, int32_t input_dtype, const float* x_ctl,
                            float* profile, float* logcounts, chm_stream_t stream);

/* The status word of chm_forward_noalloc: synchronises `stream`, then
 * returns and clears the status that the kernels of the last
 * chm_forward_noalloc calls on the current device recorded in the static
 * scratch (CHM_ERR_DEVICE_TIMEOUT when a bounded device wait gave up, else
 * CHM_OK). The counterpart of chm_read_status for callers that pass no
 * workspace; it allocates nothing either. */
int32_t chm_noalloc_read_status(chm_stream_t stream);

/* Synchronises `stream`, returns and clears the device status word that
 * the kernels of the last calls recorded in `workspace`. */
int32_t chm_read_status(void* workspace, chm_stream_t stream);

/* Self-test of the bounded device-side waits: launches one block whose
 * thread waits, with the pipelines' abortable wait (about 2 s of wall time),
 * on a barrier that nothing completes, and records the timeout in the status
 * word at `workspace` (at least 4 bytes). chm_read_status(workspace, stream)
 * then returns CHM_ERR_DEVICE_TIMEOUT; the context stays usable. No upstream
 * counterpart. */
int32_t chm_selftest_wait_timeout(void* workspace, size_t workspace_bytes,
                                  chm_stream_t stream);

/* Number of engine kernel launches the last chm_* call on this thread
 * issued (for the benchmark's launch accounting). */
int64_t chm_last_launch_count(void);

/* ---- launch timing (benchmark instrumentation) ----
 * While enabled, every engine kernel launch on the calling thread is
 * bracketed by CUDA events on its stream. chm_timing_collect synchronises
 * those events and returns, per kernel class, the summed device time (ms)
 * and launch count since the last collect; classes are
 * 0 stem, 1 stats, 2 mlp, 3 profile head, 4 count head, 5 scoring, 6 other. */
#define CHM_TIMING_CLASSES 7
void chm_timing_enable(int32_t enable);
int32_t chm_timing_collect(double* ms_per_class, int64_t* launches_per_class);

#ifdef __cplusplus
}
#endif

#endif /* CHERIMOYA_B200_H */
