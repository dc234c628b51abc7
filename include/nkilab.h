/*
 * nkilab.h - C ABI of the B200 (sm_100a) kernel set behind nkilab.ops.
 *
 * Every entry point takes caller-owned DEVICE pointers, plain integer sizes and a
 * cudaStream_t passed as `void*` (NULL = legacy default stream). Nothing here
 * allocates device memory, synchronises the stream or aborts: each call validates
 * its arguments on the host, enqueues its kernels asynchronously and returns an
 * nkl_status. nkl_last_error() gives a human-readable message for the most recent
 * failing call on the calling thread. Host-side state is limited to caches filled
 * once and then only read (per-device SM counts and kernel attributes, attention
 * work plans per shape, the device address of the static softmax scratch), each
 * behind a mutex or an atomic, so calls are thread-safe as long as callers do not
 * share output buffers or workspaces.
 *
 * Layouts are row-major and dense (the innermost dimension is contiguous):
 *   row kernels  x, y      [rows, cols]
 *   matmul       a [M, K], b [K, N], c [M, N]
 *   attention    q, k, v, out [heads, seq, head_dim]
 *
 * dtype is NKL_FLOAT32 or NKL_BFLOAT16 and applies to every tensor argument of a
 * call (inputs and output share one dtype, as in the reference, where each kernel
 * allocates its output with the input's dtype).
 *
 * Each declaration cites the reference interface it replaces, as path:line within
 * Nags-gk/nki-kernel-lab. In the reference each op is a Python function that pads /
 * transposes NumPy arrays and runs an NKI kernel on the CPU simulator; here the
 * same op is one C call over device memory.
 */
#ifndef NKILAB_H_
#define NKILAB_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NKL_ABI_VERSION 1

typedef enum nkl_status {
  NKL_OK = 0,
  NKL_ERR_SHAPE = 1,      /* a size is out of the supported range (reference: kernel assert) */
  NKL_ERR_DTYPE = 2,      /* dtype is not NKL_FLOAT32 / NKL_BFLOAT16, or unsupported for the op */
  NKL_ERR_ALIGN = 3,      /* a pointer is not aligned as the op requires (see each op) */
  NKL_ERR_CUDA = 4,       /* a CUDA runtime / driver call or kernel launch failed */
  NKL_ERR_ARG = 5,        /* NULL pointer, too-small workspace, bad flag */
  NKL_ERR_DEVICE = 7      /* a kernel reported a device-side failure (bounded wait expired) */
} nkl_status;

typedef enum nkl_dtype { NKL_FLOAT32 = 0, NKL_BFLOAT16 = 1 } nkl_dtype;

/* ---- library ------------------------------------------------------------------ */

/* ABI version (NKL_ABI_VERSION). No reference counterpart: nkilab/__init__.py:12
 * carries only a Python __version__. */
int nkl_abi_version(void);

/* Static string for a status code. */
const char* nkl_status_string(int status);

/* Message of the most recent failing call on this host thread ("" if none). */
const char* nkl_last_error(void);

/* Device-side failure flag: kernels that wait on hardware barriers give up after a
 * bounded number of polls, set this flag and return early. This call synchronises
 * `stream`, reads the flag of the current device, clears it and returns NKL_OK or
 * NKL_ERR_DEVICE. The reference has no device and no counterpart. */
int nkl_check_device(void* stream);

/* Number of SMs the persistent GEMM and attention kernels launched from the calling host
 * thread may fill (their grids and work plans size to it); 0 = all SMs, the default. The
 * tensor-parallel decoder block lowers it while its NCCL collectives run beside the GEMMs,
 * so the collectives' kernels find free SMs; results do not depend on it except through the
 * attention's split-KV plan. *previous (if not NULL) receives the value it replaces.
 * No reference counterpart (library plumbing). */
int nkl_set_sm_budget(int sms, int* previous);

/* ---- row kernels (nkilab/kernels/norm.py) ------------------------------------- */

/* y = x * rsqrt(mean(x^2) + eps) * weight, fp32 statistics, one HBM pass.
 * x, out [rows, cols]; weight [cols].
 * Replaces nkilab/ops.py:60-61 (rmsnorm) -> nkilab/kernels/norm.py:92-118 (rmsnorm_fused). */
int nkl_rmsnorm(const void* x, const void* weight, void* out, int64_t rows, int64_t cols,
                float eps, int dtype, void* stream);

/* Row softmax over the last dim, one HBM pass: y = exp(x - max) * (1 / sum).
 * Replaces nkilab/ops.py:55-57 (softmax, fused=True) -> nkilab/kernels/norm.py:65-89. */
int nkl_softmax(const void* x, void* out, int64_t rows, int64_t cols, int dtype, void* stream);

/* Bytes of device workspace nkl_softmax_unfused needs for a [rows, cols] input. */
size_t nkl_softmax_unfused_workspace_size(int64_t rows, int64_t cols);

/* Three-pass softmax that round-trips its intermediates through HBM: row max, then
 * e = exp(x - max) (fp32) with row sums, then y = e / sum. Workspace is caller-owned,
 * at least nkl_softmax_unfused_workspace_size() bytes, 256-byte aligned.
 * Replaces nkilab/ops.py:55-57 (softmax, fused=False) -> nkilab/kernels/norm.py:22-62. */
int nkl_softmax_unfused(const void* x, void* out, void* workspace, size_t workspace_bytes,
                        int64_t rows, int64_t cols, int dtype, void* stream);

/* Allocation-free variant of nkl_softmax_unfused, for callers that cannot call
 * cudaMalloc (a host that binds only this C ABI from a language runtime with no CUDA
 * allocator binding, or that must stay inside a device-memory budget owned by another
 * allocator). No counterpart in the reference, which has no device memory at all.
 * Same result as nkl_softmax_unfused; its scratch (row maxima, row sums, fp32
 * exponentials) is a fixed NKL_SOFTMAX_UNFUSED_STATIC_BYTES array in the library's
 * device image, which every GPU that loads the library holds until the process exits.
 * Inputs needing more than that (nkl_softmax_unfused_workspace_size(rows, cols) >
 * NKL_SOFTMAX_UNFUSED_STATIC_BYTES, e.g. more than about 4M fp32 elements) are
 * rejected with NKL_ERR_SHAPE and nothing is launched. The call allocates nothing.
 * The first call on each device looks up the array's device address
 * (cudaGetSymbolAddress) with that device current; make that first call before any
 * stream capture. All calls on a device share the one array and it keeps the last
 * call's contents: calls whose kernels overlap on the GPU (different streams, or
 * several host threads) race on it, so issue them on one stream. */
#define NKL_SOFTMAX_UNFUSED_STATIC_BYTES (16u * 1024u * 1024u)
int nkl_softmax_unfused_static(const void* x, void* out, int64_t rows, int64_t cols, int dtype,
                               void* stream);

/* y = silu(gate) * up, elementwise over [rows, cols], fp32 silu.
 * Replaces nkilab/ops.py:64-65 (swiglu) -> nkilab/kernels/norm.py:121-136 (swiglu_fused). */
int nkl_swiglu(const void* gate, const void* up, void* out, int64_t rows, int64_t cols,
               int dtype, void* stream);

/* ---- GEMM (nkilab/kernels/matmul.py) ------------------------------------------ */

/* c[M,N] = a[M,K] @ b[K,N], fp32 accumulation, one rounding to dtype on the way out.
 * bf16: TMA + tcgen05 tensor cores (accumulator in TMEM); requires K and N to be
 * multiples of 8 (16-byte rows for TMA) and 16-byte aligned pointers.
 * fp32: exact fp32 FMA path (no TF32), any shape.
 * Replaces nkilab/ops.py:38-52 (matmul, variant="blocked")
 *   -> nkilab/kernels/matmul.py:46-82 (matmul_blocked). */
int nkl_matmul(const void* a, const void* b, void* c, int64_t M, int64_t N, int64_t K,
               int dtype, void* stream);

/* Same product computed the way the reference's naive kernel does it: no operand
 * reuse, every (m, n, k) step reloads both tiles from global memory (plain CUDA
 * cores, fp32 accumulation). Kept as the unblocked rung of the ladder.
 * Replaces nkilab/ops.py:47-48 (matmul, variant="naive")
 *   -> nkilab/kernels/matmul.py:24-43 (matmul_naive). */
int nkl_matmul_naive(const void* a, const void* b, void* c, int64_t M, int64_t N, int64_t K,
                     int dtype, void* stream);

/* GEMM with the residual add in its epilogue: out[M, N] = residual[M, N] + a[M, K] . b[K, N],
 * bf16 only, with a . b rounded to bf16 before the add and the sum rounded once more, as
 * nkl_matmul followed by a bf16 add rounds it (so both paths give the same bits). out may
 * be residual itself. K, N multiples of 8, 16-byte-aligned pointers.
 * Replaces nkilab/model.py:89 (x + matmul(act, Wd)): the residual add after the down
 * projection, folded into the GEMM so the block makes no separate pass over it. */
int nkl_matmul_residual(const void* a, const void* b, const void* residual, void* out, int64_t M,
                        int64_t N, int64_t K, int dtype, void* stream);

/* c[M,N] = a[M,K] @ b[K,N] with bf16 a and b and the fp32 accumulator written unrounded
 * into a float c (dtype must be NKL_BFLOAT16: it names the inputs). For tensor-parallel
 * layers whose per-GPU partial products are summed across GPUs before the one rounding
 * the single-GPU product gets, so the sharded result rounds where the unsharded one does.
 * K, N multiples of 8, 16-byte-aligned pointers.
 * Replaces nkilab/kernels/matmul.py:62-79 (the fp32 PSUM accumulators before their cast on
 * copy-out) for the sharded Wo and Wd products of nkilab/model.py:86,89. */
int nkl_matmul_f32out(const void* a, const void* b, float* c, int64_t M, int64_t N, int64_t K, int dtype,
                      void* stream);

/* Fused gate/up projection with SwiGLU: out[M, F] = silu(a . Wg) * (a . Wu), bf16 only.
 * b_gate_up is [K, 2F] row-major with the columns of Wg and Wu interleaved in blocks of
 * 128 (columns 256*i .. 256*i+127 = Wg[:, 128*i ..], the next 128 = Wu[:, 128*i ..]).
 * Gate and up are rounded to bf16 before silu(gate) * up, as the unfused
 * nkl_matmul -> nkl_matmul -> nkl_swiglu path rounds them, so both paths agree.
 * F % 128 == 0, K % 8 == 0, 16-byte-aligned pointers.
 * Replaces nkilab/model.py:87-88 (swiglu(matmul(h, Wg), matmul(h, Wu))), the fusion the
 * reference lists as its next step (docs/STUDY_GUIDE.md:57). */
int nkl_matmul_swiglu(const void* a, const void* b_gate_up, void* out, int64_t M, int64_t F,
                      int64_t K, int dtype, void* stream);

/* ---- causal attention (nkilab/kernels/attention.py) --------------------------- */

/* out = softmax(q k^T * scale + causal mask) v per head, fp32 softmax statistics,
 * P rounded to dtype before the P.V product, output rounded once.
 * bf16: tcgen05 flash kernel (TMA-staged tiles, S and P.V accumulators in TMEM,
 * online softmax, fully masked key tiles skipped); head_dim 64 or 128, any seq.
 * fp32: exact fp32 flash kernel on CUDA cores; head_dim <= 128, any seq.
 * Replaces nkilab/ops.py:77-91 (attention, any "flash*" variant)
 *   -> nkilab/kernels/attention.py:155-325. */
int nkl_attention(const void* q, const void* k, const void* v, void* out, int64_t heads,
                  int64_t seq, int64_t head_dim, float scale, int dtype, void* stream);

/* Bytes of workspace nkl_attention_ws uses for this shape on the current device
 * (0 when the shape needs none: fp32, or enough query tiles to fill the GPU). */
size_t nkl_attention_workspace_size(int64_t heads, int64_t seq, int64_t head_dim, int dtype);

/* nkl_attention with a caller-owned workspace that lets the bf16 kernel split the
 * causal key range of long query tiles into chunks spread over all SMs (split-KV);
 * a second kernel on the same stream combines the partial results in a fixed chunk
 * order, so the output is bit-identical for any scheduling. The workspace
 * (>= nkl_attention_workspace_size bytes, 256-byte aligned) needs no initialisation.
 * Calls that overlap on the GPU must not share a workspace. NULL workspace or fp32:
 * same as nkl_attention.
 * Replaces nkilab/ops.py:77-91 (attention, any "flash*" variant)
 *   -> nkilab/kernels/attention.py:155-325. */
int nkl_attention_ws(const void* q, const void* k, const void* v, void* out, void* workspace,
                     size_t workspace_bytes, int64_t heads, int64_t seq, int64_t head_dim,
                     float scale, int dtype, void* stream);

/* Residual add fused with RMSNorm: sum_out = x + residual (rounded to dtype, as the
 * reference's host-side residual add in x.dtype), out = rmsnorm(sum_out, weight, eps)
 * with nkl_rmsnorm's rounding points; one pass over x and residual.
 * Replaces nkilab/model.py:86-87 (x = x + ...; rmsnorm(x, ...)), the fusion the
 * reference lists as its next step (docs/STUDY_GUIDE.md:57). */
int nkl_add_rmsnorm(const void* x, const void* residual, const void* weight, void* sum_out,
                    void* out, int64_t rows, int64_t cols, float eps, int dtype, void* stream);

/* Rotary position embedding (rotate-half convention) of x [heads, seq, head_dim] into
 * out (may equal x): for i < head_dim/2, theta_i = base^(-2i/head_dim), angle =
 * (s + pos_offset) * theta_i, out[i] = x[i] cos - x[i+d/2] sin, out[i+d/2] =
 * x[i+d/2] cos + x[i] sin, in fp32 with one rounding. head_dim a multiple of 16 (bf16)
 * or 8 (fp32), 16-byte-aligned pointers, positions below 2^24.
 * No reference counterpart: rotary embeddings are the reference's listed next step
 * (README.md:89). */
int nkl_rope(const void* x, void* out, int64_t heads, int64_t seq, int64_t head_dim, float base,
             int64_t pos_offset, int dtype, void* stream);

/* Grouped-query / multi-query attention: q, out [heads, seq, head_dim]; k, v [kv_heads,
 * seq, head_dim] with kv_heads dividing heads; query head h attends with key/value head
 * h / (heads / kv_heads). Same numerics, layouts, workspace (size from
 * nkl_attention_workspace_size(heads, ...); NULL = no split) and errors as
 * nkl_attention_ws; kv_heads == heads is plain multi-head attention.
 * No reference counterpart: GQA/MQA is the reference's listed next step (README.md:89). */
int nkl_attention_gqa(const void* q, const void* k, const void* v, void* out, void* workspace,
                      size_t workspace_bytes, int64_t heads, int64_t kv_heads, int64_t seq,
                      int64_t head_dim, float scale, int dtype, void* stream);

/* nkl_attention_gqa on strided q [heads, seq, head_dim], k and v [kv_heads, seq,
 * head_dim] and out [heads, seq, head_dim]: each is addressed as element (h, s, e) at
 * h * head_stride + s * seq_stride + e (strides in elements, positive multiples of 8,
 * i.e. 16 bytes; k and v share theirs), so q/k/v can be read straight out of a fused
 * [seq, 3, heads, head_dim] projection and out written as [seq, heads, head_dim] with no
 * transposing copies. bf16 only (NKL_ERR_DTYPE otherwise); workspace as
 * nkl_attention_ws. No reference counterpart: the reference transposes on the host
 * (nkilab/model.py:83-88). */
int nkl_attention_strided(const void* q, const void* k, const void* v, void* out, void* workspace,
                          size_t workspace_bytes, int64_t heads, int64_t kv_heads, int64_t seq,
                          int64_t head_dim, int64_t q_seq_stride, int64_t q_head_stride,
                          int64_t kv_seq_stride, int64_t kv_head_stride, int64_t out_seq_stride,
                          int64_t out_head_stride, float scale, int dtype, void* stream);

/* Launch modes of the bf16 flash kernels, the B200 rungs of the reference's flash ladder
 * (nkilab/kernels/attention.py:155-325, README.md:17-23):
 *   NKL_ATTN_AUTO             what nkl_attention_ws runs: one 128-row query tile per CTA,
 *                             Q and P in TMEM (A operands), S double buffered in TMEM, every
 *                             score row split over two warps; causal key ranges split over
 *                             all SMs where that balances the work (flash_balanced's goal)
 *   NKL_ATTN_ONE_TILE_UNSPLIT the same kernel with every query tile in one unit, no
 *                             workspace (flash / flash_kv_resident: K and V reused from L2)
 *   NKL_ATTN_TWO_TILE         two query tiles per CTA interleaved on the tensor core and two
 *                             softmax warp groups (flash_pipelined's ILP = 2 interleave);
 *                             head_dim 128, seq a multiple of 256
 *   NKL_ATTN_TWO_GROUPS       one query tile per CTA with two softmax warp groups taking
 *                             alternate key tiles (the running max handed from one to the
 *                             other), one O accumulator each, P through shared memory so S is
 *                             released as soon as it is loaded; the NKL_ATTN_AUTO split plan
 * Every mode computes the same softmax with the reference's rounding points. */
#define NKL_ATTN_AUTO 0
#define NKL_ATTN_ONE_TILE_UNSPLIT 1
#define NKL_ATTN_TWO_TILE 2
#define NKL_ATTN_TWO_GROUPS 3

/* Workspace bytes nkl_attention_mode uses for this shape and mode (0: none needed). */
size_t nkl_attention_mode_workspace_size(int64_t heads, int64_t seq, int64_t head_dim, int dtype, int mode);

/* nkl_attention_ws with an explicit launch mode (above); the same layouts, workspace rules
 * and errors, plus NKL_ERR_SHAPE when NKL_ATTN_TWO_TILE does not fit the shape.
 * Replaces nkilab/ops.py:77-91 (attention, variant=...) -> nkilab/kernels/attention.py:155-325,
 * one launch mode per rung of the reference's flash ladder. */
int nkl_attention_mode(const void* q, const void* k, const void* v, void* out, void* workspace,
                       size_t workspace_bytes, int64_t heads, int64_t seq, int64_t head_dim, float scale, int dtype,
                       int mode, void* stream);

/* Bytes of device workspace nkl_attention_naive needs: fp32 scores and dtype
 * probabilities, each [heads, seq, seq]. */
size_t nkl_attention_naive_workspace_size(int64_t heads, int64_t seq, int dtype);

/* Unfused attention that materialises the masked score matrix (fp32) and the
 * normalised probabilities (dtype) in HBM, then multiplies by v.
 * Replaces nkilab/ops.py:77-91 (attention, variant="naive")
 *   -> nkilab/kernels/attention.py:35-89 (attention_naive). */
int nkl_attention_naive(const void* q, const void* k, const void* v, void* out,
                        void* workspace, size_t workspace_bytes, int64_t heads, int64_t seq,
                        int64_t head_dim, float scale, int dtype, void* stream);

/* ---- head-sharded attention with its all-gather over NVLink ----------------------- */

/* Device memory several processes of one node map (CUDA IPC), for the all-gather below:
 * nkl_ipc_alloc allocates `bytes` (zeroed) on the current device and writes its
 * nkl_ipc_handle_bytes()-byte handle; another process opens the handle with nkl_ipc_open
 * (a pointer valid on its current device, peer access enabled) and releases it with
 * nkl_ipc_close; the owner frees it with nkl_ipc_free once no process uses it.
 * No reference counterpart (the reference runs on one NeuronCore). */
size_t nkl_ipc_handle_bytes(void);
int nkl_ipc_alloc(size_t bytes, void** ptr, void* handle);
int nkl_ipc_open(const void* handle, void** ptr);
int nkl_ipc_close(void* ptr);
int nkl_ipc_free(void* ptr);

/* Causal attention of this GPU's heads, gathered into every GPU's output in the same call:
 * q, k, v [heads, seq, head_dim] bf16 are this rank's heads, which are heads
 * [head_offset, head_offset + heads) of the full [heads_total, seq, head_dim] output.
 * outs[r] is rank r's output buffer and flags[r] rank r's flag array (world + 1 uint32,
 * zeroed before the first call), as pointers valid on this device (nkl_ipc_open for the
 * other ranks'). The attention kernel stores each finished output tile into every rank's
 * buffer over NVLink (TMA stores; split tiles' merge kernel writes every buffer too), then a
 * one-warp kernel exchanges per-call counts through the flag arrays (system-scope release /
 * acquire, bounded wait: NKL_ERR_DEVICE from nkl_check_device if a peer never arrives), so
 * when the call's work on `stream` completes, every rank's heads are in this rank's buffer.
 * Every rank must make the same sequence of calls. A rank writes into the others' buffers
 * while they may still read the previous call's result, so alternate two buffer sets
 * between consecutive calls (the second-previous call's readers on every rank have finished
 * when the previous call's count exchange completes). workspace as nkl_attention_ws for
 * (heads, seq, head_dim). world <= 8, bf16, head_dim 64 or 128.
 * Replaces nkilab/ops.py:77-91 (attention) for the head sharding and output gather the
 * B200 build adds; the reference has no distributed code. */
int nkl_attention_allgather(const void* q, const void* k, const void* v, void* const* outs,
                            unsigned int* const* flags, int world, int rank, int64_t heads_total,
                            int64_t head_offset, void* workspace, size_t workspace_bytes, int64_t heads,
                            int64_t seq, int64_t head_dim, float scale, int dtype, void* stream);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* NKILAB_H_ */
