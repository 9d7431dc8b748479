/*
 * cobra_b200.h -- C ABI of the B200 (sm_100a) single transformer-layer forward.
 *
 * The reference (dalberrt/COBRA-GPU-Kernel, torch_transformer_benchmark.py) is
 * pure Python: its drop-in is the nn.Module ``UserOptimizedTransformer``
 * (:917-1541) whose forward drives Triton kernels. This header is the native
 * boundary underneath the equivalent module of this repository; every entry
 * point names the reference function it replaces.
 *
 * Conventions
 *   - Plain pointers are device pointers on the current CUDA device unless
 *     stated otherwise. ``stream`` is a cudaStream_t passed as void*.
 *   - Every call is asynchronous on ``stream``, allocates nothing, never
 *     synchronises the host, and is safe to capture in a CUDA graph.
 *   - Return value: B200L_OK (0) or a negative B200L_ERR_* code; the message
 *     of the last failure on the calling thread is available through
 *     b200l_last_error().
 *   - Device-side failures (a pipeline wait that exceeded its time limit) are
 *     recorded in the status word at the start of the workspace and read with
 *     b200l_read_status(); kernels never trap.
 *
 * Layout (T = batch*seq_len tokens, d = d_model, H heads, dh = d/H,
 * dhp = dh rounded up to 32/64/128/256):
 *   x, y      fp32 [T, d] row-major (the reference's [B,S,d] tensors)
 *   wqkv      fp16 [3d, d]  rows q(0..d-1), k(d..2d-1), v(2d..3d-1); nn.Linear
 *             weight layout, i.e. K-major (torch_transformer_benchmark.py:876-883)
 *   bqkv      fp32 [3d]
 *   wo        fp16 [d, d];  bo fp32 [d]
 *   ln*_w/_b  fp32 [d]
 *   workspace 1024-byte aligned, every region 1024-aligned (sp = S rounded
 *             up to 8); b200l_kernel_workspace_bytes gives the full layout
 *             [status 256 B][q fp16 B*H*S*dhp][k fp16 B*H*S*dhp]
 *             [v^T fp16 B*H*dhp*sp][ctx fp16 T*d][h fp16 T*d, only d > 256],
 *             b200l_layer_workspace_bytes what b200l_layer_forward needs (the
 *             status block alone when the whole-layer kernel runs)
 */
#ifndef COBRA_B200_H
#define COBRA_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define B200L_API __attribute__((visibility("default")))
#else
#define B200L_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define B200L_ABI_VERSION 4

enum b200l_status {
    B200L_OK = 0,
    B200L_ERR_BAD_SHAPE = -1,          /* non-positive size, d % H != 0, d > 2048, aliasing */
    B200L_ERR_UNSUPPORTED_HEAD_DIM = -2, /* d/H not a multiple of 32 in [32, 256] */
    B200L_ERR_NULL_POINTER = -3,
    B200L_ERR_WORKSPACE_TOO_SMALL = -4,
    B200L_ERR_LAUNCH = -5,             /* a CUDA launch or attribute call failed */
    B200L_ERR_DEVICE = -6,             /* not an sm_100 device */
    B200L_ERR_TIMEOUT = -7,            /* a device pipeline wait ran out (status word) */
    B200L_ERR_ALIGNMENT = -8           /* a pointer is not 16-byte aligned */
};

/* Layer description. Replaces the per-layer state the reference keeps in
 * ``_LayerPack`` (torch_transformer_benchmark.py:857-914) plus the shape and
 * policy fields ``_prepare`` derives (:948-1081). */
typedef struct b200l_layer_desc {
    int32_t batch;        /* B */
    int32_t seq_len;      /* S */
    int32_t d_model;      /* d <= 2048 */
    int32_t num_heads;    /* H, d % H == 0, d/H a multiple of 32 in [32, 256] */
    int32_t causal;       /* 0: full attention (the judged mode), 1: causal */
    float eps1;           /* norm1 eps (nn.LayerNorm default 1e-5) */
    float eps2;           /* norm2 eps */
    const void* wqkv;     /* fp16 [3d, d] */
    const float* bqkv;    /* fp32 [3d] */
    const void* wo;       /* fp16 [d, d] */
    const float* bo;      /* fp32 [d] */
    const float* ln1_w;   /* fp32 [d] */
    const float* ln1_b;
    const float* ln2_w;
    const float* ln2_b;
    /* Optional key-padding mask, uint8 [B, S] (a torch bool tensor's bytes;
     * nonzero = valid token), or NULL for none. As in BaselineSelfAttention
     * (torch_transformer_benchmark.py:106-109, :121-122) and the fused path's
     * attn_bias / row mask (:1201-1214): invalid keys get probability 0 in
     * every query's softmax, and an invalid query row's attention output
     * (after the out-projection and its bias) is zeroed, so that row of y is
     * LN2(x). Read by the attention and out-projection kernels. */
    const uint8_t* valid_mask;
    /* Head sharding (0 = every head, the normal case). When 0 < local_heads
     * <= num_heads, K1 and K2 (b200l_qkv_ln_gemm, b200l_flash_attn) compute
     * only local_heads heads: wqkv / bqkv hold those heads' rows (their q
     * rows, then their k rows, then their v rows, each local_heads * dh), and
     * ctx in the workspace is [T, local_heads * dh]. The out-projection mixes
     * every head (torch_transformer_benchmark.py:119), so b200l_outproj_res_ln,
     * b200l_layer_forward and b200l_block_forward need local_heads == 0: a
     * head-sharded caller gathers every rank's ctx columns first (see
     * headshard.py in the package). */
    int32_t local_heads;
} b200l_layer_desc;

/* ABI version (B200L_ABI_VERSION). */
B200L_API int b200l_version(void);

/* Copies the last error message of the calling thread into buf (NUL-terminated,
 * truncated to n bytes); returns the length of the full message. */
B200L_API int b200l_last_error(char* buf, size_t n);

/* Bytes of workspace b200l_layer_forward needs for this description, by the
 * path it takes: 1024 (the status block alone) when the whole-layer kernel
 * runs (d_model 64 or 128, head_dim 32, seq_len <= 128), else the status block
 * and every intermediate (as b200l_kernel_workspace_bytes). 0 for a bad shape.
 * Replaces the reference's live-set estimate ``_activation_bytes_per_seq``
 * (torch_transformer_benchmark.py:1364-1400), but exact. */
B200L_API size_t b200l_layer_workspace_bytes(const b200l_layer_desc* desc);

/* Bytes of workspace the per-kernel entry points (b200l_qkv_ln_gemm,
 * b200l_flash_attn, b200l_outproj_res_ln) need: the status block and every
 * intermediate of the layout above. Same reference counterpart as
 * b200l_layer_workspace_bytes (:1364-1400). */
B200L_API size_t b200l_kernel_workspace_bytes(const b200l_layer_desc* desc);

/* Zeroes the status word at the start of a workspace (async on stream). */
B200L_API int b200l_clear_status(void* workspace, void* stream);

/* Reads the status word (synchronises ``stream``): 0 when no kernel recorded a
 * failure, else the B200L_ERR_* code that was recorded. */
B200L_API int b200l_read_status(const void* workspace, void* stream);

/* Test hook for the bounded-wait path (no counterpart in the reference, whose
 * only failure handling is the eager fallback after a failed graph capture,
 * torch_transformer_benchmark.py:1527-1534). Arms, in the workspace's status
 * block (async on ``stream``), a fault site and a per-wait time limit that
 * every later kernel on this workspace reads at its start:
 *   site B200L_DEBUG_SITE_ATTN_KV: in CTA 0 of the attention kernel for
 *     head_dim <= 64, the TMA producer leaves out its first K / v^T load;
 *   site B200L_DEBUG_SITE_GEMM_OPERAND: in CTA 0 of the TMA-fed GEMM (the
 *     out-projection; also the QKV projection for d_model > 256), the
 *     producer leaves out its first operand load.
 * The consumer's wait for that stage then runs out after wait_limit_ns
 * (0 = the normal 2 s; otherwise at least 1 ms), the CTA unwinds (every copy
 * it issued is drained, its TMEM is freed), and B200L_ERR_TIMEOUT is recorded
 * for b200l_read_status. Nothing faults, traps or hangs. b200l_clear_status
 * disarms it. */
#define B200L_DEBUG_SITE_NONE 0
#define B200L_DEBUG_SITE_ATTN_KV 1
#define B200L_DEBUG_SITE_GEMM_OPERAND 2
B200L_API int b200l_debug_arm(void* workspace, int32_t site, uint64_t wait_limit_ns, void* stream);

/* Packs nn.Linear weights into the layout above: wqkv = cast_fp16(cat(wq, wk,
 * wv)), bqkv = cat(bq, bk, bv), wo16 = cast_fp16(wo). Inputs fp32 on device.
 * Replaces ``_LayerPack.__init__`` (torch_transformer_benchmark.py:873-914). */
B200L_API int b200l_pack_weights(int32_t d_model, const float* wq, const float* wk, const float* wv,
                       const float* bq, const float* bk, const float* bv, const float* wo,
                       void* wqkv16, float* bqkv32, void* wo16, void* stream);

/* The whole layer: y = LN2(x + Attn(LN1(x)) Wo^T + bo). x and y must not alias.
 * Replaces ``UserOptimizedTransformer._run_fused`` for one layer
 * (torch_transformer_benchmark.py:1170-1327: lines 1216-1223, 1227-1238,
 * 1262-1268) and, as the module's forward, ``forward`` (:1512-1541). */
B200L_API int b200l_layer_forward(const b200l_layer_desc* desc, const float* x, float* y,
                        void* workspace, size_t ws_bytes, void* stream);

/* The per-kernel entry points below need a workspace of
 * b200l_kernel_workspace_bytes (every intermediate).
 *
 * K1: h = LN1(x) fused into the QKV projection on tcgen05; writes q, k
 * ([B,H,S,dhp] fp16) and v^T ([B,H,dhp,S] fp16) into the workspace.
 * Replaces ``_tl_add_ln`` (:539-569, used at :1220-1223) + ``F.linear``/
 * ``_gemm_kernel`` for qkv (:283-381, :1234). */
B200L_API int b200l_qkv_ln_gemm(const b200l_layer_desc* desc, const float* x,
                      void* workspace, size_t ws_bytes, void* stream);

/* K2: ctx = softmax(q k^T / sqrt(dh)) v per (batch, head), flash-style on
 * tcgen05, scores never written to memory; reads q/k/v^T from the workspace
 * and writes ctx fp16 [T, d] into it. Replaces ``_tl_attn``/``_attn_kernel``
 * (:572-649, :828-854) and the SDPA fallback (:1239-1253). */
B200L_API int b200l_flash_attn(const b200l_layer_desc* desc, void* workspace, size_t ws_bytes,
                     void* stream);

/* K3: y = LN2(x + ctx Wo^T + bo) on tcgen05 with the residual and LayerNorm in
 * the epilogue (for d > 256 the epilogue stores the residual and a row
 * LayerNorm pass follows). Replaces ``_tl_linear_ln``/``_gemm_ln_kernel``
 * (:394-488, used at :1262-1268). */
B200L_API int b200l_outproj_res_ln(const b200l_layer_desc* desc, const float* x, float* y,
                         void* workspace, size_t ws_bytes, void* stream);

/* Full encoder block, for stacks that include the reference's GELU FFN:
 *   x1 = x + Attn(LN1(x)); y = x1 + W2 gelu_erf(W1 LN2(x1) + b1) + b2,
 * padded rows of y zeroed (valid_mask). The attention half uses the layer
 * kernels; the FFN half is two tcgen05 GEMMs (bias + exact GELU to fp16 in the
 * first epilogue, bias + residual + row mask in the second).
 * Replaces BaselineTransformerBlock.forward (torch_transformer_benchmark.py:
 * 135-146) as the reference's fused path computes it (:1274-1292: _tl_linear
 * with resid, _tl_add_ln, _tl_linear gelu=True, _tl_linear with rmask). */
typedef struct b200l_block_desc {
    b200l_layer_desc layer;  /* attention half, norm1, norm2 (eps2 is norm2's) */
    int32_t ffn_dim;         /* f, a positive multiple of 8 */
    const void* w1;          /* fp16 [f, d]  ffn_in.weight */
    const float* b1;         /* fp32 [f]     ffn_in.bias */
    const void* w2;          /* fp16 [d, f]  ffn_out.weight */
    const float* b2;         /* fp32 [d]     ffn_out.bias */
} b200l_block_desc;

/* Workspace bytes of b200l_block_forward: the layer workspace, then the fp32
 * residual x1 [T, d], LN2(x1) fp16 [T, d] and the FFN hidden fp16 [T, f]. */
B200L_API size_t b200l_block_workspace_bytes(const b200l_block_desc* desc);

B200L_API int b200l_block_forward(const b200l_block_desc* desc, const float* x, float* y,
                                  void* workspace, size_t ws_bytes, void* stream);

/* y = LayerNorm(x) row by row (fp32 in/out, d a multiple of 4, at most 2048),
 * rows whose row_mask byte is 0 set to zero (row_mask may be NULL). x may equal
 * y. The stack's final_norm and its padded-row mask: replaces
 * BaselineTransformer.forward :170-172 (fused as _tl_add_ln mask_out, :1289-1291). */
B200L_API int b200l_row_layernorm(const float* x, float* y, const float* w, const float* b, float eps,
                                  int64_t rows, int32_t d, const uint8_t* row_mask, void* stream);

/* dst = fp16(src) for n elements: packs nn.Linear weights for the FFN GEMMs.
 * Replaces the fp16 weight copies of _LayerPack (torch_transformer_benchmark.py:
 * 873-914) for ffn_in / ffn_out. */
B200L_API int b200l_cast_f16(const float* src, void* dst, int64_t n, void* stream);

/* dst = src converted between element types (round to nearest even), n
 * elements, both 16-byte aligned: the boundary conversion that lets the fp32
 * layer take and return fp16 / bf16 tensors (the reference's
 * --dtype float16 / bfloat16 harness modes, torch_transformer_benchmark.py:
 * 952-962, :1091-1094, run the same layer in that dtype). */
#define B200L_DTYPE_F32 0
#define B200L_DTYPE_F16 1
#define B200L_DTYPE_BF16 2
B200L_API int b200l_convert(const void* src, int32_t src_type, void* dst, int32_t dst_type, int64_t n,
                            void* stream);

/* Allocation-free variant of b200l_layer_forward. No counterpart in the
 * reference (its Python module always allocates through PyTorch).
 *
 * For callers that cannot call cudaMalloc: a plugin whose host process owns
 * all device memory through its own pool, or a latency-critical service that
 * forbids allocation after start-up (cudaMalloc/cudaFree synchronise the
 * device). The scratch the kernels need comes from a fixed array of
 * B200L_NOALLOC_MAX_SCRATCH_BYTES inside the library, which every GPU that
 * loads the library holds until exit; problems whose workspace
 * (b200l_layer_workspace_bytes) exceeds it are rejected with
 * B200L_ERR_WORKSPACE_TOO_SMALL. The caller still passes x and y.
 *   - The first call on each device looks up the array's device address
 *     (cudaGetSymbolAddress, with that device current); make that first call
 *     before any stream capture.
 *   - Nothing is allocated or freed; the status block at the start of the
 *     array is cleared (cudaMemsetAsync) at the start of every call.
 *   - All calls on a device share the one array and it keeps the last call's
 *     contents: calls that overlap on the GPU (different streams without
 *     ordering between them) race and corrupt each other's results.
 *   - A device-side failure (B200L_ERR_TIMEOUT) of a call is recorded in the
 *     array's status block: read it with b200l_noalloc_read_status before the
 *     next no-alloc call on that device, which clears it.
 *   - The device address is looked up once per device and kept for the life
 *     of the process; do not call this entry point on a device again after a
 *     cudaDeviceReset of it. */
#define B200L_NOALLOC_MAX_SCRATCH_BYTES (64u * 1024u * 1024u)
B200L_API int b200l_layer_forward_noalloc(const b200l_layer_desc* desc, const float* x, float* y,
                                          void* stream);

/* Status of the last b200l_layer_forward_noalloc call(s) on the current
 * device, as b200l_read_status reads a workspace (synchronises ``stream``): 0,
 * or the B200L_ERR_* code a kernel recorded. No counterpart in the reference
 * (see b200l_layer_forward_noalloc). */
B200L_API int b200l_noalloc_read_status(void* stream);

#ifdef __cplusplus
}
#endif

#endif /* COBRA_B200_H */
