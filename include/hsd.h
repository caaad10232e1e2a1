/*
 * hsd.h -- C ABI of libhsd.so, the sm_100a (B200) implementation of the sparse MoE
 * down-projection hot path of mlx-heimr-sparse-down.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t passed as
 * `void*`; none allocates, synchronises the device or reads back to the host, so all
 * of them are stream-ordered and can be captured in a CUDA graph -- except the one-time
 * set-up calls of expert parallelism (hsd_ep_alloc / free / ipc_* / set_peers) and
 * hsd_device_status, which say so. Every entry point
 * returns an hsd_status; on failure hsd_last_error_string() (thread-local) says why.
 * No entry point aborts the process and no kernel traps: a bad index met on the device
 * is skipped and recorded in a per-device status word read by hsd_device_status().
 *
 * Layouts (affine 4-bit, group 64, the mlx-lm convention):
 *   checkpoint  w [.., D, F/8] u32 (8 nibbles of one output row per word, low nibble
 *               first), s / b [.., D, F/64] (bf16 or f16), W[o, i] = s*q + b
 *   neuron-major (after hsd_to_neuron_major)
 *               pw [.., F, D/8] u32: row i = neuron i, word w packs W[8w .. 8w+7, i]
 *               ps / pb [.., F/64, D]
 *
 * Each declaration names the reference function it replaces (path:line inside the
 * mlx-heimr-sparse-down project).
 */
#ifndef HSD_H
#define HSD_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* status codes (the reference's only error channel is a Python assert,
 * hsd/model.py:147,234,249, and MSL static_asserts, hsd/decode.py:50-51) */
enum {
  HSD_OK = 0,
  HSD_ERR_SHAPE = 1,   /* a size the kernels do not support */
  HSD_ERR_ALIGN = 2,   /* a pointer not aligned as the kernel needs */
  HSD_ERR_DTYPE = 3,   /* an unsupported dtype code */
  HSD_ERR_CUDA = 4,    /* a CUDA runtime call failed */
  HSD_ERR_TIMEOUT = 5, /* a bounded device-side wait ran out */
  HSD_ERR_NCCL = 6,    /* reserved for the expert-parallel exchange */
  HSD_ERR_ARG = 7,     /* a null pointer or an out-of-range argument */
  HSD_ERR_INDEX = 8    /* (device status word) an expert id outside [0, E) */
};

/* dtype codes */
enum { HSD_F32 = 0, HSD_F16 = 1, HSD_BF16 = 2 };

/* ---- library state ------------------------------------------------------------ */

/* The message of the last failed call on this host thread ("" when none). */
const char* hsd_last_error_string(void);

/* ABI version of this header (bumped on any signature change). */
int hsd_abi_version(void);

/* Reads and clears the calling device's status word (HSD_OK or the first
 * device-side error code recorded since the last read). Synchronises `stream`. */
int hsd_device_status(int* status_out, void* stream);

/* ---- layout: hsd/layout.py -------------------------------------------------- */

/* hsd/layout.py:34 nibble_transpose(w):
 *   w [lead, R, CW] u32 -> out [lead, 8*CW, R/8] u32 with out[.., c, wo] packing
 *   W[8*wo + n, c], n = 0..7, low nibble first. Exact and self-inverse.
 *   R must be a multiple of 8. out must not alias w. */
int hsd_nibble_transpose(const uint32_t* w, uint32_t* out, int64_t lead, int64_t R,
                         int64_t CW, void* stream);

/* hsd/layout.py:72-73 (the scales / biases half of to_neuron_major):
 *   in [lead, R, C] 16-bit -> out [lead, C, R] (swapaxes(-1, -2), bit-exact). */
int hsd_swap_last2_u16(const uint16_t* in, uint16_t* out, int64_t lead, int64_t R,
                       int64_t C, void* stream);

/* ---- decode: hsd/decode.py ---------------------------------------------------- */

/* hsd/decode.py:164 sparse_down(h, sel, gains, pw, ps, pb, spw, sps, spb, *, F, FS, D,
 * topk, sl, unr, nds, out_dtype, loadsc):
 *   h     [B, topk*F + FS] (h_dtype: bf16 / f16 / f32), the ReLU^2 activations of the
 *         selected experts then the shared expert's
 *   sel   [B, topk] int32 routed expert ids in [0, E)
 *   gains [B, topk+1] f32 (routing scores, then the shared expert's gain)
 *   pw    [E, F, D/8] u32, ps / pb [E, F/64, D] (s_dtype: bf16 / f16)
 *   spw   [FS, D/8] u32,   sps / spb [FS/64, D]
 *   resid [B, D] (y_dtype) or NULL: when given, y = resid + down(h)
 *   y     [B, D] (y_dtype: bf16 / f16 / f32)
 * Reads only the weight rows of nonzero h entries and the scales / biases of 64-neuron
 * groups with at least one nonzero entry. loadsc = 0 is the reference's benchmark-only
 * switch (hsd/decode.py:25-27) that skips the scale / bias loads.
 * topk = 0 (the shared expert alone; sel / pw / ps / pb may be NULL, gains [B, 1]) and FS = 0
 * (routed experts alone; spw / sps / spb may be NULL) are the per-slot forms the
 * expert-parallel exchange uses.
 * Supported: D % 32 == 0, F % 64 == 0, FS % 64 == 0, 1 <= B <= 65535; h, pw, ps, pb, spw,
 * sps and spb 16-byte aligned (HSD_ERR_ALIGN otherwise). Launched with programmatic
 * dependent launch: it waits for the previous kernel in the stream before reading. */
int hsd_sparse_down_decode(const void* h, int h_dtype, const int32_t* sel,
                           const float* gains, const uint32_t* pw, const void* ps,
                           const void* pb, int s_dtype, const uint32_t* spw,
                           const void* sps, const void* spb, const void* resid, void* y,
                           int y_dtype, int B, int D, int F, int FS, int topk, int E,
                           int loadsc, void* stream);

/* The dense form of the same kernel: every row of the selected experts is read (the
 * down projection of hsd/model.py:132-133 decode_dense) on the neuron-major layout, with
 * the sparse kernel's own fixed reduction order -- a row whose h is zero adds an exact zero
 * where the sparse form skips it, so hsd_sparse_down_decode reproduces this output bit for
 * bit on any input. No counterpart in the reference (its dense path is mlx-lm's stock
 * gather_qmm); it is the exact-parity reference of the sparse form. Same arguments as
 * hsd_sparse_down_decode without loadsc. */
int hsd_dense_down_decode_nm(const void* h, int h_dtype, const int32_t* sel, const float* gains,
                             const uint32_t* pw, const void* ps, const void* pb, int s_dtype,
                             const uint32_t* spw, const void* sps, const void* spb,
                             const void* resid, void* y, int y_dtype, int B, int D, int F, int FS,
                             int topk, int E, void* stream);

/* The active-index sets of the decode kernel (hsd/decode.py:86-101): per (token, slot),
 * slot < topk routed and slot == topk the shared expert, the ascending indices of the
 * nonzero h entries, compacted by the same warp-ballot routine the decode kernel runs.
 *   live  [B, topk+1, max(F, FS)] int32 (entries past the count are left untouched)
 *   count [B, topk+1] int32 */
int hsd_decode_live_rows(const void* h, int h_dtype, int32_t* live, int32_t* count, int B,
                         int F, int FS, int topk, void* stream);

/* ---- prefill: hsd/prefill.py --------------------------------------------------- */

/* The fixed tile count of build_tiles (hsd/prefill.py:266,275): nt_routed =
 * T*topk/tt + E (a bound that every routing meets), nt_shared = ceil(T/tt). Host-only, no
 * device work. */
int hsd_prefill_num_tiles(int T, int topk, int E, int tt, int* nt_routed, int* nt_shared);

/* hsd/prefill.py:247 build_tiles(sel, E, tt):
 *   sel [T, topk] int32 -> tile_e [NT] int32 (expert, E = shared, -1 = empty),
 *   tile_slot [NT*tt] int32 (slot t*topk+k for routed tiles, token t for shared tiles,
 *   -1 padding), NT = nt_routed + nt_shared. Inside an expert, slots keep ascending order.
 *   E <= 256. An expert id outside [0, E) is recorded in the status word and its slot dropped. */
int hsd_prefill_build_tiles(const int32_t* sel, int T, int topk, int E, int tt, int32_t* tile_e,
                            int32_t* tile_slot, void* stream);

/* hsd/prefill.py:281 build_union(h, tile_e, tile_slot, *, F, FS, topk, E, tt, kc, nth):
 *   ulist [NT, umax] int32: per tile the ascending union of the columns nonzero in any of
 *   its slots (-1 padded), ucount [NT] int32. umax >= max(F, FS); tt <= 1024. */
int hsd_prefill_build_union(const void* h, int h_dtype, const int32_t* tile_e,
                            const int32_t* tile_slot, int NT, int tt, int F, int FS, int topk,
                            int E, int umax, int32_t* ulist, int32_t* ucount, void* stream);

/* Workspace bytes hsd_sparse_down_prefill needs for (T, D, F, FS, topk, E): one live byte per
 * (tile, 64-neuron group), the gathered fp16 A rows of every tile and the fp32 partial rows
 * [T*(topk+1), D]. Host-only. */
int hsd_prefill_workspace_bytes(int T, int D, int F, int FS, int topk, int E, size_t* bytes);

/* hsd/prefill.py:294 sparse_down_prefill(h, sel, gains, pw, ps, pb, spw, sps, spb, *, F, FS,
 * D, topk, E, tt, nb, kc, nsg, tiles, union, out_dtype):
 *   h [T, topk*F+FS], gains [T, topk+1] f32, tiles from hsd_prefill_build_tiles with
 *   tt = 128, layouts as for decode -> y [T, D] (+ resid). Gathers the tiles' h rows (fp16),
 *   runs the tcgen05 grouped GEMM (weights dequantised to fp16 in shared memory, fp32
 *   accumulation in TMEM, routing gain in the epilogue; a K-tile -- 64 neurons -- with no
 *   nonzero h in any of the tile's slots is skipped, hsd/prefill.py:11-16's union at group
 *   granularity) and sums each token's topk+1
 *   partial rows in a fixed order. The caller provides `workspace` (16-byte aligned) of at
 *   least hsd_prefill_workspace_bytes(). Supported: D % 192 == 0, F % 64 == 0, FS % 64 == 0. */
int hsd_sparse_down_prefill(const void* h, int h_dtype, const float* gains, const int32_t* tile_e,
                            const int32_t* tile_slot, int NT, const uint32_t* pw, const void* ps,
                            const void* pb, int s_dtype, const uint32_t* spw, const void* sps,
                            const void* spb, const void* resid, void* y, int y_dtype, int T, int D,
                            int F, int FS, int topk, int E, void* workspace, size_t workspace_bytes,
                            void* stream);

/* ---- Mamba-2 verify / rollback: hsd/mamba.py ------------------------------------- */

/* The causal-conv half of hsd/mamba.py:28-32 (mamba_verify): window = [conv_state; conv_in]
 * (K-1+L rows, conv_state NULL = zeros) is copied to `padded` (conv_in's dtype) and
 * out[t, c] = silu(bias[c] + sum_j w[c, j] * window[t + j, c]) in fp32. conv_in rows are
 * in_stride elements apart (a slice of the in_proj output). L >= 1, K == 4.
 * in_dtype f32 / bf16, w_dtype f32 / bf16, out_dtype f32 / f16 / bf16. */
int hsd_mamba_conv_verify(const void* conv_in, int in_dtype, int64_t in_stride,
                          const void* conv_state, const void* w, int w_dtype, const void* bias,
                          void* out, int out_dtype, void* padded, int L, int C, int K, void* stream);

/* The SSM half of hsd/mamba.py:33-41 (mamba_verify with mlx-lm's ssm_update) for L rows:
 *   xbc [L, >= H*P + 2*G*N] (x | B | C per row, x_dtype f32 / bf16, rows xbc_stride apart),
 *   dt [L, >= H] (dt_dtype f32 / bf16, rows dt_stride apart), A_log / D / dt_bias [H] f32,
 *   state0 [H, P, N] f32 (NULL = zeros) -> y [L, H*P] (y_dtype f32 / bf16) and
 *   states [L, H, P, N] f32: the state after every row (the per-row checkpoints).
 * dt_t = clamp(softplus(dt + dt_bias), dt_min, dt_max). Rows run as single steps would, so
 * states[n-1] equals n single steps bit for bit. last_only != 0 (a prefill chunk, never rolled
 * back): only the final state, in states[0] ([1, H, P, N]). N in {32, 64, 128, 256}, H % G == 0. */
int hsd_mamba_ssm_verify(const void* xbc, int x_dtype, int64_t xbc_stride, const void* dt,
                         int dt_dtype, int64_t dt_stride, const float* A_log, const float* D,
                         const float* dt_bias, float dt_min, float dt_max, const float* state0,
                         float* states, void* y, int y_dtype, int L, int H, int P, int G, int N,
                         int last_only, void* stream);

/* hsd/mamba.py:47 mamba_rollback(records, n_keep), on device and without recomputation:
 * state_out = states[n_keep-1], conv_out = padded[n_keep : n_keep+K-1] (elem_bytes per
 * element), one copy kernel. 1 <= n_keep <= L; states and state_out 16-byte aligned and
 * H*P*N % 4 == 0 (HSD_ERR_ALIGN otherwise). */
int hsd_mamba_rollback(const float* states, const void* padded, int elem_bytes, int n_keep, int L,
                       int H, int P, int N, int C, int K, float* state_out, void* conv_out,
                       void* stream);

/* Resident-buffer forms of the two verify kernels, for decode loops replayed from a CUDA
 * graph (no counterpart in the reference, whose rollback re-runs ssm_update over the kept
 * rows, hsd/mamba.py:47-56). The previous call's outputs are the inputs: the conv window is
 * padded[*n_keep .. *n_keep+K-2] and the SSM state states[*n_keep-1], where *n_keep (device
 * memory, 1 <= *n_keep <= rows) is the number of rows the previous call kept -- 1 after a
 * plain step, a+1 after a verify whose first a drafts were accepted. The call writes the
 * window and its L new rows to padded[0 .. K-2+L] and the state after each row to
 * states[0 .. L-1], in place. padded [rows + K - 1, C] (zeros before the first call),
 * states [rows, H, P, N] fp32 (zeros before the first call), 1 <= L <= rows. A *n_keep
 * outside 1..rows is read as 1 and recorded as HSD_ERR_INDEX in the status word. */
int hsd_mamba_conv_step(const void* conv_in, int in_dtype, int64_t in_stride, void* padded,
                        const int* n_keep, int rows, const void* w, int w_dtype, const void* bias,
                        void* out, int out_dtype, int L, int C, int K, void* stream);

int hsd_mamba_ssm_step(const void* xbc, int x_dtype, int64_t xbc_stride, const void* dt,
                       int dt_dtype, int64_t dt_stride, const float* A_log, const float* D,
                       const float* dt_bias, float dt_min, float dt_max, float* states,
                       const int* n_keep, int rows, void* y, int y_dtype, int L, int H, int P,
                       int G, int N, void* stream);

/* ---- MoE front end (the caller of the down kernel) -------------------------------- */

/* hsd/model.py:110-121 front(): the routed up projections (mlx gather_qmm of fc1 over the
 * selected experts) and the shared expert's up_proj, each followed by relu2, fused into one
 * launch that writes the down kernel's input directly:
 *   h[b, k*F + f]    = relu(sum_d Wu[sel[b,k]][f, d] * x[b, d])^2   for k < topk, f < F
 *   h[b, topk*F + f] = relu(sum_d Wsu[f, d] * x[b, d])^2             for f < FS
 * Up weights in the checkpoint layout along the hidden axis: uw [E, F, D/8] u32, us / ub
 * [E, F, D/64] (s_dtype); suw [FS, D/8], sus / sub [FS, D/64]. x [B, D] with row stride
 * x_stride elements; h [B, topk*F + FS] contiguous. On the tensor cores (mma.m16n8k16): x
 * rounded to fp16 (exact for bf16 inside fp16's range), the nibbles as exact fp16 integers,
 * fp32 accumulation, one rounding to h_dtype; a token's outputs do not depend on the other
 * tokens of the call. D % 64 == 0, D <= 8192, uw / suw 16-byte aligned; topk == 0 (shared only) and
 * FS == 0 (routed only) are allowed. An expert id outside [0, E) gives zeros for that slot
 * and HSD_ERR_INDEX in the status word. */
int hsd_moe_up_decode(const void* x, int x_dtype, int64_t x_stride, const int32_t* sel,
                      const uint32_t* uw, const void* us, const void* ub, int s_dtype,
                      const uint32_t* suw, const void* sus, const void* sub, void* h,
                      int h_dtype, int B, int D, int F, int FS, int topk, int E, void* stream);

/* hsd/model.py:132-133 decode_dense (the stock path: mlx gather_qmm of fc2 over the
 * selected experts and the shared expert's down_proj), as the sparse kernel's comparison
 * point on the same device: every weight of the selected experts is read from the checkpoint
 * layout (w [E, D, F/8], s / b [E, D, F/64]; sw [D, FS/8], ss / sb [D, FS/64]), fp32
 * accumulation, the part's gain applied, the partial rows written to part [B, topk+1, D]
 * fp32 (caller-owned workspace) and summed in slot order (+ resid) into y [B, D]. Same
 * h / sel / gains / resid / y conventions as hsd_sparse_down_decode. D % 32 == 0, F and FS
 * multiples of 64 and <= 8192, w / sw 16-byte aligned. */
int hsd_dense_down_decode(const void* h, int h_dtype, const int32_t* sel, const float* gains,
                          const uint32_t* w, const void* s, const void* b, int s_dtype,
                          const uint32_t* sw, const void* ss, const void* sb, const void* resid,
                          void* y, int y_dtype, float* part, int B, int D, int F, int FS, int topk,
                          int E, void* stream);

/* The model's other 4-bit linears at decode (mlx QuantizedLinear, the layers around the hot
 * path: Mamba in / out projections, attention projections, lm_head), on the tensor cores as
 * hsd_moe_up_decode (the weights read once for up to 8 rows, a row's result independent of
 * the other rows):
 *   y[b, o] = (resid[b, o] +) sum_i W[o, i] * x[b, i]
 * w [out_f, in_f/8] u32, s / b [out_f, in_f/64] (s_dtype); x [B, in_f] with row stride
 * x_stride; resid (may be NULL) and y [B, out_f] contiguous in y_dtype. x in fp16, fp32
 * accumulation, the residual added in fp32, one rounding. in_f % 64 == 0, in_f <= 8192, w
 * 16-byte aligned. */
int hsd_qlinear_decode(const void* x, int x_dtype, int64_t x_stride, const uint32_t* w, const void* s,
                       const void* b, int s_dtype, const void* resid, void* y, int y_dtype, int B,
                       int in_f, int out_f, void* stream);

/* ---- per-row operators of the decode step (the model around the hot path) --------- */

/* RMSNorm as NemotronH applies it (mlx.fast.rms_norm in the reference's model): per row
 * y = w * cast(x * rsqrt(mean(x^2) + eps)), the normalised row rounded to x's dtype before
 * the weight multiply, fp32 arithmetic. x [B, D] with row stride x_stride; y [B, D]. */
int hsd_rms_norm(const void* x, int x_dtype, int64_t x_stride, const void* w, int w_dtype, void* y,
                 int y_dtype, int B, int D, float eps, void* stream);

/* The Mamba-2 mixer's gated norm: g = y * silu(gate), per group of `group` channels
 * out = w * cast(g * rsqrt(mean(g^2) + eps)). y [B, I] (row stride y_stride), gate [B, I]
 * (row stride g_stride), out [B, I] contiguous. I % group == 0. */
int hsd_gated_rms_norm(const void* y, int y_dtype, int64_t y_stride, const void* gate, int g_dtype,
                       int64_t g_stride, const void* w, int w_dtype, void* out, int out_dtype, int B,
                       int I, int group, float eps, void* stream);

/* The MoE router (hsd/model.py:115, the block's gate): scores = sigmoid(x . R_e) in fp32 for
 * R [E, D] fp32, the top-k experts by score (ties to the lower id) -> sel [B, topk] int32 and
 * gains [B, topk+1] f32 = the scores over their sum, then 1 for the shared expert.
 * scores [B, E] fp32 is scratch; ticket is one caller-owned unsigned int, zero before the
 * first call and reset by every call (calls sharing a ticket must not overlap).
 * 1 <= topk <= min(E, 16), E <= 1024, B <= 65535. */
int hsd_router_topk(const void* x, int x_dtype, int64_t x_stride, const float* R, int B, int D, int E,
                    int topk, float* scores, unsigned int* ticket, int32_t* sel, float* gains,
                    void* stream);

/* The attention of decode rows over a fixed-size cache (the reference model's GQA block at
 * decode, mlx-lm nemotron_h, no positional encoding), for steps replayed from a captured
 * graph: the position is read on the device. q [L, QH*HD] bf16 (row stride q_stride,
 * a multiple of 8), kc / vc [KVH, max_len, HD] bf16 with rows pos .. pos+L-1 already
 * written, *pos (device int64) the tokens before row 0; row l attends keys 0 .. pos+l with
 * scale `scale` -> out [L, QH*HD] bf16. ws: fp32 workspace of
 * hsd_attn_decode_workspace_bytes(L, QH, max_len) bytes. HD 64 or 128, QH/KVH <= 16. A row's
 * result does not depend on the other rows of the call. pos + L > max_len is clamped and
 * recorded as HSD_ERR_INDEX in the status word. */
int hsd_attn_decode_workspace_bytes(int L, int QH, int max_len, size_t* bytes);
int hsd_attn_decode(const void* q, int64_t q_stride, const void* kc, const void* vc,
                    const int64_t* pos, void* out, float* ws, int L, int QH, int KVH, int HD,
                    int max_len, float scale, void* stream);

/* ---- allocation-free prefill ------------------------------------------------------ */

/* No counterpart in the reference. For callers that cannot call cudaMalloc (code running
 * under CUDA graph capture without a memory pool, runtimes that own all device memory,
 * hosts that must not grow device memory after start-up): the same computation as
 * hsd_sparse_down_prefill, with its scratch in one fixed device array inside this library
 * (hsd_prefill_noalloc_max_bytes() bytes, 64 MiB, held by every GPU that loads the library
 * until exit) instead of a caller workspace. The caller still passes inputs and outputs,
 * tiles built with tt = 128. A call whose scratch would exceed the array returns
 * HSD_ERR_SHAPE with the bytes it needs (at the reference shapes: up to about 11 tokens;
 * a model with fewer experts or narrower layers admits more). The first call on a device
 * looks up the array's device address (cudaGetSymbolAddress) with that device current;
 * make that first call before any stream capture. hsd_prefill_noalloc_max_bytes does the
 * same look-up for the current device (when one is present), so calling it once per device
 * does the set-up without inputs. Calls share the array: calls whose work
 * overlaps on the GPU (different streams or host threads) race; calls ordered on one
 * stream do not. Allocates nothing, frees nothing. */
int hsd_prefill_noalloc_max_bytes(size_t* bytes);
int hsd_sparse_down_prefill_noalloc(const void* h, int h_dtype, const float* gains,
                                    const int32_t* tile_e, const int32_t* tile_slot, int NT,
                                    const uint32_t* pw, const void* ps, const void* pb,
                                    int s_dtype, const uint32_t* spw, const void* sps,
                                    const void* spb, const void* resid, void* y, int y_dtype,
                                    int T, int D, int F, int FS, int topk, int E, void* stream);

/* ---- expert parallelism over the GPUs of one box ----------------------------------- */

/* The MoE down projection with the routed experts sharded round robin over `world` GPUs
 * (expert e on rank e % world, local index e / world), the shared expert replicated and
 * every token on its home rank: a multi-GPU form of hsd/decode.py:164 sparse_down and
 * hsd/prefill.py:294 sparse_down_prefill (the reference has one GPU). One process per GPU.
 * The exchange is this library's own: every rank's INBOX (hsd_ep_alloc memory, mapped into
 * the other ranks' processes with the IPC calls below) is written by the others with plain
 * stores over NVLink, ordered by release/acquire flags at system scope; no collective
 * library, no multicast, nothing read back to the host (a call can be captured in a CUDA
 * graph). A call is hsd_ep_dispatch, then hsd_ep_expert, then hsd_ep_combine, on one stream;
 * every rank makes the same calls in the same order with the same (world, max_tokens, topk,
 * F, D, E); B may differ between ranks and may be 0. One inbox and workspace serve every
 * call and every layer of a rank. Every device-side wait for another rank is bounded by
 * timeout_s (<= 0: 10 s); running out records HSD_ERR_TIMEOUT in the status word, the call's
 * output is unspecified and the ranks must allocate their buffers again. */
#define HSD_EP_IPC_HANDLE_BYTES 64

/* Bytes of a rank's inbox and of its private workspace (256-byte aligned, from any
 * allocator). n_local: the routed experts the rank holds (<= 0: E / world); the inbox does
 * not depend on it. At world 8, max_tokens 512 and the reference shapes: 130 MB and 203 MB. */
int hsd_ep_buffer_bytes(int world, int max_tokens, int topk, int F, int FS, int D, int E,
                        int n_local, size_t* inbox_bytes, size_t* workspace_bytes);
/* Zeroed device memory that other processes can map (cudaMalloc; free with hsd_ep_free).
 * The one allocation this library makes, and only here. */
int hsd_ep_alloc(size_t bytes, void** ptr);
int hsd_ep_free(void* ptr);
/* The HSD_EP_IPC_HANDLE_BYTES-byte handle of hsd_ep_alloc memory, its mapping in another
 * process (with peer access enabled), and the unmapping. */
int hsd_ep_ipc_handle(const void* ptr, void* handle);
int hsd_ep_ipc_open(const void* handle, void** ptr);
int hsd_ep_ipc_close(void* ptr);
/* Stores the inboxes of ranks 0..world-1 as this process addresses them (its own included)
 * in the workspace; once, before the first call. Synchronises the stream. */
int hsd_ep_set_peers(void* workspace, const uint64_t* inbox_addrs, int world, void* stream);
/* Routes this rank's B tokens: hcat [B, topk*F + FS] (bf16 or f16, 16-byte aligned), sel
 * [B, topk] int32 global expert ids, gains [B, topk+1] f32. Each (token, slot) row goes to its
 * expert's owner with its local id and gain. emap (device, [E] int32, this rank's table, or
 * NULL for round robin: owner e % world, local id e / world): emap[e] = owner << 16 | local id
 * at the owner; an expert replicated on every rank maps to this rank itself. An id outside
 * [0, E), or a table entry naming no rank, is recorded as HSD_ERR_INDEX and the slot
 * contributes nothing defined. */
int hsd_ep_dispatch(void* workspace, int rank, int world, int max_tokens, const void* hcat,
                    int h_dtype, const int32_t* sel, const float* gains, int B, int topk, int F,
                    int FS, int D, int E, const int32_t* emap, double timeout_s, void* stream);
/* The GEMM side: the slots this rank received times its n_local experts pw [n_local, F, D/8],
 * ps / pb [n_local, F/64, D] (neuron-major, s_dtype bf16 or f16, local-id order; n_local <= 0:
 * E / world), and the shared
 * expert spw [FS, D/8], sps / spb [FS/64, D] of this rank's own B tokens (the same hcat as the
 * dispatch), in one tensor-core GEMM launch; each fp32 partial row times its gain is stored
 * into its home rank's inbox. inbox: this rank's own inbox. */
int hsd_ep_expert(void* workspace, void* inbox, int rank, int world, int max_tokens,
                  const void* hcat, int h_dtype, int B, const uint32_t* pw, const void* ps,
                  const void* pb, const uint32_t* spw, const void* sps, const void* spb,
                  int s_dtype, int topk, int F, int FS, int D, int E, int n_local, double timeout_s,
                  void* stream);
/* y [B, D] f32 = the sum over each token's topk partial rows in slot order, then its shared
 * expert row (FS > 0). */
int hsd_ep_combine(void* workspace, int rank, int world, int max_tokens, float* y, int B,
                   int topk, int F, int FS, int D, int E, double timeout_s, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* HSD_H */
