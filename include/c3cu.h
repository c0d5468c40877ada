/*
 * c3cu.h — C ABI of the B200 (sm_100a) kernels behind the C3 fused hot path.
 *
 * Every entry point is `extern "C"`, takes plain device pointers, sizes and an explicit
 * CUDA stream (`c3cu_stream_t` is a cudaStream_t; 0 = the legacy default stream), launches
 * asynchronously and returns an int status: C3CU_OK (0) or a negative C3CU_ERR_* code.
 * No C++ exception and no torch type crosses this boundary. The message of the last
 * failure on the calling thread is available from c3cu_last_error().
 *
 * Layouts are row-major. "bf16" buffers hold IEEE bfloat16 (uint16_t bit patterns),
 * "f32" buffers IEEE binary32. Pointers handed to the tensor-core entry points must be
 * 16-byte aligned and their row strides multiples of 16 bytes (TMA rule); violations are
 * reported as C3CU_ERR_ALIGN before anything is launched.
 *
 * Reference interface each entry point replaces (ShengFlow/C3, file:line):
 *   c3cu_linear_bias_relu_fwd  <- the region kernel of "MatMul+Add+ReLU": MultiNodeKernelFunc
 *                                 c3_kernel(inputs{X,B,b}, out, n, M, K, N, scratch)
 *                                 (include/C3/C3KernelRegistry.h:80; built by
 *                                 src/C3/MLIRKernelGen.cpp:783-1253, installed by
 *                                 include/C3/C3HotPathManager.h:799-929)
 *   c3cu_relu_mask_db          <- ReLU backward Mul(Gt(x,0),grad) (src/C3/C3BackwardCapture.cpp:501-528)
 *                                 fused with Add backward SumReduce axis 0
 *                                 (src/C3/C3BackwardCapture.cpp:618-644; src/C3/C3DialectLowering.cpp:382-465)
 *   c3cu_gemm_dx / c3cu_gemm_dw <- MatMul backward grad@B^T and A^T@grad
 *                                 (src/C3/C3BackwardCapture.cpp:681-723) executed through
 *                                 C3KernelRegistry::tryExecuteBackward (src/C3/C3KernelRegistry.cpp:230-322)
 *   c3cu_gemm_bf16             <- c3.matmul with transA/transB folding (src/C3/C3DialectLowering.cpp:467-610)
 *   c3cu_ew_chain_cfg4 /
 *   c3cu_ew_program            <- FusedNode elementwise loops (src/C3/MLIRKernelGen.cpp:394-768) and
 *                                 LinalgFusedKernel (src/C3/LinalgFusedGen.cpp:141-378)
 *   c3cu_sum_rows_f32          <- SumReduceOpLowering axis 0 (src/C3/C3DialectLowering.cpp:382-465)
 *   c3cu_flash_attn_fwd        <- no reference counterpart (the reference has no attention kernel;
 *                                 op::Softmax exists only as a rolling-hash code,
 *                                 src/C3/RollingHash.cpp:62)
 */
#ifndef C3CU_H_
#define C3CU_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef void* c3cu_stream_t;

#define C3CU_OK 0
#define C3CU_ERR_INVALID (-1)     /* null pointer, negative or unsupported size */
#define C3CU_ERR_ALIGN (-2)       /* TMA alignment rule violated */
#define C3CU_ERR_CUDA (-3)        /* CUDA runtime / driver error */
#define C3CU_ERR_FAULT (-4)       /* a kernel recorded a fault (bounded wait gave up) */
#define C3CU_ERR_UNSUPPORTED (-5) /* no sm_100 device current */
#define C3CU_ERR_WORKSPACE (-6)   /* workspace missing or too small */

#define C3CU_DTYPE_F32 0
#define C3CU_DTYPE_BF16 1

/* Weight layouts accepted by the Linear entry points. */
#define C3CU_W_NK 0 /* W[N][K] (nn.Linear): Y = X * W^T */
#define C3CU_W_KN 1 /* B[K][N] (the reference's MatMul rhs): Y = X * B */

/* GEMM epilogues for c3cu_gemm_bf16. */
#define C3CU_EPI_BIAS_RELU_MASK 0 /* out bf16 = max(acc+bias,0), mask bit = (acc+bias > 0) */
#define C3CU_EPI_STORE_BF16 1
#define C3CU_EPI_STORE_F32 2
#define C3CU_EPI_BIAS_STORE_F32 3

/* ------------------------------------------------------------------ library status */
int c3cu_version(void);
const char* c3cu_last_error(void);
/* C3CU_OK when the current CUDA device is an sm_100 (B200-class) part. */
int c3cu_device_check(void);
/* Reads (and clears) the fault words the kernels write when a bounded wait gives up.
 * Synchronises the device. *code = 0 when no kernel recorded a fault. */
int c3cu_fault_status(uint32_t* code);

/* ------------------------------------------------------------------ Linear+bias+ReLU
 * Forward of the MatMul+Add+ReLU region: Y = max(X*W^T + b, 0) (C3CU_W_NK) or
 * Y = max(X*B + b, 0) (C3CU_W_KN); bf16 inputs, fp32 accumulation, bf16 output.
 * mask: [M][ceil(N/32)] uint32, bit j of word w = (pre-activation[m][32w+j] > 0). */
int c3cu_linear_bias_relu_fwd(const void* X, const void* W, const float* bias, void* Y,
                              uint32_t* mask, int64_t M, int64_t N, int64_t K, int w_layout,
                              c3cu_stream_t stream);

/* Backward pre-pass: dZ = dY * mask (bf16, exact) and db[n] = sum_m dZ[m][n] (fp32).
 * Needs a device workspace of c3cu_relu_mask_db_workspace(M, N) bytes for the partial
 * column sums; calls that may run at the same time (different streams) need different
 * workspaces. The first call on a (device, stream) allocates a 256 KiB array of reduction
 * tickets that the library keeps for that stream (the tickets return to zero after every
 * call, so later calls launch only the kernel). The same holds for c3cu_sum_rows_f32. */
size_t c3cu_relu_mask_db_workspace(int64_t M, int64_t N);
int c3cu_relu_mask_db(const void* dY, const uint32_t* mask, void* dZ, float* db, int64_t M,
                      int64_t N, void* workspace, size_t workspace_bytes, c3cu_stream_t stream);

/* The same pre-pass for callers that cannot allocate device memory: a host framework whose
 * allocator owns every byte of device memory and forbids side allocations, or a latency-
 * critical path where cudaMalloc's implicit device synchronisation is unacceptable. No
 * counterpart exists in the reference (its CPU kernels take a host scratch pointer).
 * Scratch is a fixed array of C3CU_NOALLOC_SCRATCH_BYTES in device memory that the library
 * owns (every GPU that loads the library holds it until exit); the call needs
 * c3cu_relu_mask_db_workspace(M, N) <= C3CU_NOALLOC_SCRATCH_BYTES (for N = 4096 up to
 * M = 130560 rows) and returns C3CU_ERR_WORKSPACE beyond that. It allocates nothing. Its
 * first call on a device looks up the array's device address, so make that first call
 * before any stream capture; after a cudaDeviceReset the next call looks it up again (the
 * reloaded library's array may sit elsewhere), so make that call outside a capture too.
 * M = 0 writes db = 0. All calls share the one array: calls that overlap on the GPU
 * (concurrent streams, or several host threads) race and must be serialised by the caller. */
#define C3CU_NOALLOC_SCRATCH_BYTES (4 * 1024 * 1024)
int c3cu_relu_mask_db_noalloc(const void* dY, const uint32_t* mask, void* dZ, float* db,
                              int64_t M, int64_t N, c3cu_stream_t stream);

/* dX = dZ * W (C3CU_W_NK, W[N][K]) or dZ * B^T (C3CU_W_KN, B[K][N]); bf16 out [M][K]. */
int c3cu_gemm_dx(const void* dZ, const void* W, void* dX, int64_t M, int64_t N, int64_t K,
                 int w_layout, c3cu_stream_t stream);

/* dW = dZ^T * X as fp32 [N][K] (C3CU_W_NK) or dB = X^T * dZ as fp32 [K][N] (C3CU_W_KN). */
int c3cu_gemm_dw(const void* dZ, const void* X, float* dW, int64_t M, int64_t N, int64_t K,
                 int w_layout, c3cu_stream_t stream);

/* General tensor-core GEMM: out[M][N] = epi(A * B^T) with
 *   A: a_mn == 0 -> stored [M][lda] (K contiguous); a_mn == 1 -> stored [K][lda] (M contiguous)
 *   B: b_mn == 0 -> stored [N][ldb] (K contiguous); b_mn == 1 -> stored [K][ldb] (N contiguous)
 * out row stride ldo (elements), mask row stride ldm (words). */
int c3cu_gemm_bf16(const void* A, int64_t lda, int a_mn, const void* B, int64_t ldb, int b_mn,
                   void* out, int64_t ldo, int epilogue, const float* bias, uint32_t* mask,
                   int64_t ldm, int64_t M, int64_t N, int64_t K, c3cu_stream_t stream);

/* Cap on the CTAs of the persistent tensor-core GEMMs that the CALLING THREAD launches from now
 * on (0 = one per SM, the default). A host that overlaps a collective with a GEMM lowers it
 * around that launch to leave SMs free; GEMMs launched by other threads are not affected. */
int c3cu_set_gemm_max_ctas(int max_ctas);
/* CTAs per thread-block cluster of the in-switch all-reduce launches that follow (process-wide):
 * 1 (the default) or 2. With 2 (and an even num_ctas) each pair of CTAs runs on the two SMs of
 * one TPC, so a CTA-pair GEMM running beside the all-reduce keeps whole TPCs. */
int c3cu_set_collective_cluster(int ctas_per_cluster);
/* GEMM kernel variant for the calls that follow (process-wide): 0 = automatic (the CTA-pair
 * kernel, 256 x 256 tiles on two SMs with cta_group::2, whenever M > 128, else the single-CTA
 * 128 x 256 kernel; when the last wave of tiles would leave half of the SM pairs idle, its
 * tiles are split in two K halves whose fp32 partial sums are added once, K-half order
 * fixed), 1 = single-CTA kernel only, 2 = CTA-pair kernel without the K split. Variants 1
 * and 2 give identical bits (the same K order); on split tiles variant 0 accumulates the two
 * K halves separately, so it differs from them within the fp32 accumulation error bound.
 * The first split launch on a (device, stream) allocates a 21 MB workspace (fp32 partials and
 * tickets) that the library keeps for that stream; capture such a launch in a CUDA graph only
 * after one uncaptured call on the same stream. */
int c3cu_set_gemm_variant(int variant);
/* Limit, in nanoseconds, on the wait of a split-K tile's second half for the first half's
 * fp32 partial (process-wide, for launches that follow; 0 restores the default of 4 s). A
 * test shortens it to make that wait run out, which records C3CU_ERR_FAULT (read with
 * c3cu_fault_status) without faulting the GPU: the recovery path of a split GEMM whose partner
 * was late. After c3cu_fault_status reports a fault, the next split launch on each stream
 * clears its workspace first. No counterpart in the reference (its kernels never wait). */
int c3cu_set_split_wait_ns(uint64_t ns);
/* Programmatic dependent launch for the GEMM and pre-pass kernels (process-wide; 0 = off, the
 * default): each such kernel may be scheduled while the previous kernel on its stream drains,
 * runs its prologue (barrier initialisation, TMEM allocation, descriptor prefetch) and then
 * waits for that kernel's completion before it touches global memory. Results are unchanged. */
int c3cu_set_launch_overlap(int enable);
/* Per-shape variant table filled by a tuner (the B200 counterpart of the reference's tile
 * auto-tuner, include/C3/AutoTuner.h:42-63, src/C3/C3Engine.cpp:1577-1651): calls of exactly
 * (M, N, K, a_mn, b_mn, epilogue) use `variant` instead of the process-wide one. */
int c3cu_gemm_tune_set(int64_t M, int64_t N, int64_t K, int a_mn, int b_mn, int epilogue, int variant);
int c3cu_gemm_tune_get(int64_t M, int64_t N, int64_t K, int a_mn, int b_mn, int epilogue, int* variant);
int c3cu_gemm_tune_clear(void);

/* ------------------------------------------------------------------ exact fp32 (CUDA cores)
 * Bit-exact restatements of the reference's fp32 loops: every output element is reduced
 * over k in ascending order with separate round-to-nearest multiply and add.
 * c3cu_matmul_f32: out[M][N] = act(bias-init + sum_k a(i,k) b(k,j)) with
 *   a(i,k) = transA ? A[k*M+i] : A[i*K+k],  b(k,j) = transB ? B[j*K+k] : B[k*N+j],
 *   bias-init = bias ? bias[bias_numel == 1 ? 0 : j] : 0,  act: 0 none, 1 ReLU, 2 sigmoid, 3 tanh
 *   (c3.matmul, src/C3/C3DialectLowering.cpp:467-610).
 * c3cu_region_fwd_f32: T = sum (from 0); s = T + bias[idx % bias_numel]; out = max(s, 0);
 *   z (optional) = s; mask (optional) as in c3cu_linear_bias_relu_fwd
 *   (MatMul + FusedNode{Add, ReLU}, src/C3/MLIRKernelGen.cpp:610-768). */
int c3cu_matmul_f32(const float* A, const float* B, float* out, int64_t M, int64_t K, int64_t N,
                    int transA, int transB, const float* bias, int64_t bias_numel, int act,
                    c3cu_stream_t stream);
int c3cu_region_fwd_f32(const float* X, const float* B, const float* bias, int64_t bias_numel,
                        float* out, float* z, uint32_t* mask, int64_t M, int64_t K, int64_t N,
                        int transB, c3cu_stream_t stream);
/* The captured backward of two chained regions, fused pairwise, bit-exact:
 * c3cu_matmul_relu_bwd_f32: out = (z > 0 ? 1 : 0) * (sum_k a(i,k) b(k,j)) -- MatMul backward dA
 *   (grad @ B^T, src/C3/C3BackwardCapture.cpp:681-723) followed by the upstream ReLU's backward
 *   Mul(Gt(z, 0), .) (:501-528); z [M][N] is that ReLU's input.
 * c3cu_matmul_colsum_f32: out[M][N] = sum_k a(i,k) b(k,j) and colsum[j] = sum_k b(k,j) in k order
 *   -- MatMul backward dB (A^T @ grad) with the Add backward's SumReduce of grad (:618-644,
 *   src/C3/C3DialectLowering.cpp:382-465), both from one pass over grad.
 * Operand indexing, transposes and the k order as in c3cu_matmul_f32. */
int c3cu_matmul_relu_bwd_f32(const float* A, const float* B, const float* z, float* out, int64_t M, int64_t K,
                             int64_t N, int transA, int transB, c3cu_stream_t stream);
int c3cu_matmul_colsum_f32(const float* A, const float* B, float* out, float* colsum, int64_t M, int64_t K,
                           int64_t N, int transA, int transB, c3cu_stream_t stream);
/* Column sums in the reference's order (rows ascending), bit-exact; no workspace. */
int c3cu_sum_rows_f32_exact(const float* in, float* out, int64_t M, int64_t N,
                            c3cu_stream_t stream);

/* ------------------------------------------------------------------ elementwise chains
 * The chain relu((A + B) * C - A) / (1 + exp(-B)) over n fp32 elements, one pass. */
int c3cu_ew_chain_cfg4(const float* A, const float* B, const float* C, float* out, int64_t n,
                       c3cu_stream_t stream);

/* General single-pass chain. `code` holds n_instr instructions of 4 bytes
 * {opcode, dst, src0, src1} over 16 fp32 registers; registers 0..n_inputs-1 are loaded
 * from inputs[i][idx % numels[i]] (numels[i] == n: no broadcast), and register `out_reg`
 * is stored to out[idx]. Opcodes: see C3CU_EW_* below. */
#define C3CU_EW_MAX_INPUTS 8
#define C3CU_EW_MAX_INSTR 64
#define C3CU_EW_MAX_OUTPUTS 4
#define C3CU_EW_ADD 1
#define C3CU_EW_SUB 2
#define C3CU_EW_MUL 3
#define C3CU_EW_DIV 4        /* plain IEEE division */
#define C3CU_EW_DIV_NANZ 5   /* division returning NaN when the divisor is 0 */
#define C3CU_EW_NEG 6
#define C3CU_EW_RELU 7       /* maxnum(x, 0) */
#define C3CU_EW_EXP 8
#define C3CU_EW_LOG 9
#define C3CU_EW_SIGMOID 10   /* 1 / (1 + exp(-x)) */
#define C3CU_EW_TANH 11      /* tanh(x) */
#define C3CU_EW_TANH_EXP 12  /* (exp(x) - exp(-x)) / (exp(x) + exp(-x)) */
#define C3CU_EW_GT 13        /* src0 > src1 ? 1 : 0 (ordered: NaN -> 0) */
#define C3CU_EW_CONST 14     /* dst = constant table[src0] */
#define C3CU_EW_MOV 15
int c3cu_ew_program(const float* const* inputs, const int64_t* numels, int n_inputs,
                    const uint8_t* code, int n_instr, const float* constants, int n_constants,
                    int out_reg, float* out, int64_t n, c3cu_stream_t stream);

/* out[i] = in[i] converted between C3CU_DTYPE_F32 and C3CU_DTYPE_BF16 (round to nearest even). */
/* The same register machine with up to C3CU_EW_MAX_OUTPUTS outputs: outs[j] receives
 * register out_regs[j], all from one pass over the inputs. */
int c3cu_ew_program_multi(const float* const* inputs, const int64_t* numels, int n_inputs,
                          const uint8_t* code, int n_instr, const float* constants, int n_constants,
                          const int* out_regs, float* const* outs, int n_out, int64_t n,
                          c3cu_stream_t stream);

/* Fused backward of a chain of unary elementwise nodes (the reference's fused backward
 * sequences, src/C3/C3BackwardCapture.cpp:874-1637), one pass over n fp32 elements.
 * node_ops[k] (k = 0 is the most downstream node, the first in backward order) is one of
 * C3CU_BW_*; xs[k] is that node's forward input (unused for Neg); outs[k] receives the
 * gradient node k passes upstream, i.e. the input gradient of node k + 1. */
#define C3CU_BW_RELU 1
#define C3CU_BW_SIGMOID 2
#define C3CU_BW_TANH 3
#define C3CU_BW_NEG 4
#define C3CU_BW_EXP 5
#define C3CU_BW_LOG 6
#define C3CU_BW_MAX_CHAIN 4
int c3cu_ew_backward_chain(const int* node_ops, int n_nodes, const float* grad, const float* const* xs,
                           float* const* outs, int64_t n, c3cu_stream_t stream);

int c3cu_convert(const void* in, int in_dtype, void* out, int out_dtype, int64_t n,
                 c3cu_stream_t stream);

/* db[n] = sum over rows of a fp32 matrix [M][N] (axis 0), deterministic order. */
size_t c3cu_sum_rows_f32_workspace(int64_t M, int64_t N);
int c3cu_sum_rows_f32(const float* in, float* out, int64_t M, int64_t N, void* workspace,
                      size_t workspace_bytes, c3cu_stream_t stream);

/* ------------------------------------------------------------------ attention
 * FlashAttention forward: O = softmax(scale * Q K^T (+ causal mask)) V, bf16 in/out,
 * fp32 accumulation; LSE[b][h][s] = natural-log sum of exp of the scaled, masked scores
 * (may be NULL). Q, K, V, O: [B][H][S][D] contiguous bf16 with D = 128. */
int c3cu_flash_attn_fwd(const void* Q, const void* K, const void* V, void* O, float* LSE,
                        int64_t B, int64_t H, int64_t S, int64_t D, float scale, int causal,
                        c3cu_stream_t stream);
/* Attention kernel for the calls that follow (process-wide): 0 = default (3); 1 = one
 * 128-row query tile per CTA; 2 = two query tiles per CTA sharing each 128-key K / V block;
 * 3 = two query tiles per CTA, 64-key blocks with two S buffers per tile in TMEM; 4 = 3 with
 * the two tiles' softmax warps taking turns at their exponentials (experimental). */
int c3cu_set_attn_variant(int variant);

/* ------------------------------------------------------------------ fused dW GEMM + all-reduce
 * The data-parallel backward's exchange step fused into the dW GEMM that produces it (replaces
 * the dW graph of MatMul backward, src/C3/C3BackwardCapture.cpp:681-723, followed by a sum over
 * ranks; the reference runs one process and has no collective):
 *   dW[N][K] = sum over ranks of dZ_r^T X_r   (bf16 out, fp32 accumulation, one rounding per
 *                                              rank, fp32 accumulation of the ranks' partials
 *                                              in the NVSwitch)
 *   db[n]    = sum over ranks of db_r[n]       (fp32, in place)
 * dZ_r [M][N] and X_r [M][K] are this rank's rows (M may differ per rank, M >= 1). dW is this
 * rank's copy of a buffer that every rank bound to one NVLink multicast object, mc_dW its
 * multicast address; mc_db the multicast address of this rank's db_r (db_count fp32, a multiple
 * of 4; 0 for none); flags / mc_flags this rank's copy and the multicast address of
 * C3CU_AR_FLAG_WORDS(N, K) uint32 words in multicast memory, zero before the first call. Every
 * rank makes the same sequence of calls with epoch = 0, 1, 2, ... When the call completes on
 * the stream, dW and db hold the sums on every rank. Each tile of dW is reduced as soon as all
 * ranks have computed it, while later tiles are still on the tensor cores. Waits for other
 * ranks are bounded (2 s) and record C3CU_ERR_FAULT. world == 1 runs the plain dW GEMM. */
#define C3CU_AR_FLAG_WORDS(N, K) (4 + 16 * ((((N) + 255) / 256) * (((K) + 255) / 256)))
int c3cu_gemm_dw_allreduce(const void* dZ, const void* X, void* dW, void* mc_dW, float* mc_db,
                           int64_t db_count, uint32_t* flags, uint32_t* mc_flags, int64_t flag_words,
                           int64_t M, int64_t N, int64_t K, int rank, int world, uint32_t epoch,
                           c3cu_stream_t stream);

/* ------------------------------------------------------------------ data-parallel collective
 * In-switch (NVLink SHARP) all-reduce (sum) of fp32 elements [lo, hi) of a buffer that every
 * rank has bound to one NVLink multicast object. mc_data / mc_flag are the multicast
 * addresses of the data and of a uint32 barrier counter in the same buffer, local_flag
 * this rank's own copy of that counter (zero on every rank before the first call). Every
 * rank calls with the same lo, hi, num_ctas and epoch (0, 1, 2, ... per call). Waits on
 * peers are bounded; a rank that never arrives makes the kernel record a fault
 * (c3cu_fault_status) and return. The dW/db all-reduce of the data-parallel training step
 * uses it; the reference has no collective. */
int c3cu_nvls_allreduce_f32(float* mc_data, uint32_t* mc_flag, const uint32_t* local_flag,
                            int64_t lo, int64_t hi, int rank, int world, uint32_t epoch,
                            int num_ctas, c3cu_stream_t stream);
/* The same protocol over two segments of one multicast buffer in one call: bf16_count bf16
 * elements at byte offset bf16_offset (summed in the switch with fp32 accumulation, one
 * rounding to bf16) and f32_count fp32 elements at f32_offset. Offsets are multiples of 16
 * bytes, bf16_count of 8 and f32_count of 4. */
int c3cu_nvls_allreduce(void* mc_base, uint32_t* mc_flag, const uint32_t* local_flag,
                        int64_t bf16_offset, int64_t bf16_count, int64_t f32_offset, int64_t f32_count,
                        int rank, int world, uint32_t epoch, int num_ctas, c3cu_stream_t stream);
/* c3cu_nvls_allreduce with the bf16 segment split in two parts that run at once on disjoint
 * CTAs: elements [0, bf16_peer_from) and the fp32 segment are summed in the switch by
 * num_ctas - peer_ctas CTAs; elements [bf16_peer_from, bf16_count) by peer_ctas CTAs that read
 * their rank's slice from every rank's copy through its unicast address, add in fp32 in rank
 * order, round once to bf16 and broadcast with multimem.st. peer_bases is a host array of
 * `world` (at most 8) 16-byte-aligned device addresses: rank r's copy of the buffer as mapped in
 * this process (its own copy at [rank]). bf16_peer_from is a multiple of 8; peer_ctas is 0 when
 * the peer part is empty and otherwise leaves at least one CTA for a non-empty switch part.
 * Same barrier counter and epoch sequence as c3cu_nvls_allreduce (one epoch per call). */
int c3cu_nvls_allreduce_split(void* mc_base, const void* const* peer_bases, uint32_t* mc_flag,
                              const uint32_t* local_flag, int64_t bf16_offset, int64_t bf16_count,
                              int64_t bf16_peer_from, int64_t f32_offset, int64_t f32_count, int rank,
                              int world, uint32_t epoch, int num_ctas, int peer_ctas, c3cu_stream_t stream);

/* ------------------------------------------------------------------ training step (cfg1)
 * Softmax cross-entropy over C classes, mean over B rows, fp32, one kernel:
 *   lse_i = m_i + log(sum_c exp(z[i][c] - m_i)),  m_i = max_c z[i][c]  (c ascending)
 *   *loss = (sum_i (lse_i - z[i][labels[i]])) / B   (i ascending for B <= 8192)
 *   dlogits[i][c] = (exp(z[i][c] - lse_i) - (c == labels[i])) * (1 / B)   (may be NULL)
 * A label outside [0, C) makes the loss and that row of dlogits NaN. The reference trains
 * with its host framework's loss, which is not part of its sources: textbook definition. */
int c3cu_softmax_ce_f32(const float* logits, const int32_t* labels, float* loss, float* dlogits,
                        int64_t B, int64_t C, c3cu_stream_t stream);
/* Plain SGD over `count` (1..C3CU_SGD_MAX_TENSORS) fp32 tensors in one launch:
 * params[t][i] = params[t][i] - lr * grads[t][i] (multiply, then subtract; no FMA). */
#define C3CU_SGD_MAX_TENSORS 8
int c3cu_sgd_f32(float* const* params, const float* const* grads, const int64_t* numels, int count,
                 float lr, c3cu_stream_t stream);

/* Gradient all-reduce (sum, in place) through an NCCL communicator: `count` elements of
 * `dtype` (C3CU_DTYPE_F32 or C3CU_DTYPE_BF16) at `grads` on `stream`. `comm` is an
 * ncclComm_t, e.g. from c3cu_nccl_comm_init, whose id rank 0 made with c3cu_nccl_unique_id
 * (128 bytes) and the host passed to every rank. NCCL is loaded at run time ("libnccl.so.2",
 * the copy already in the process if any); without it these calls return
 * C3CU_ERR_UNSUPPORTED. This is the exchange step of the data-parallel training step, named
 * in the hot path's C ABI (dW || db after c3cu_gemm_dw / c3cu_relu_mask_db); the reference
 * itself has no collective. */
int c3cu_nccl_version(int* version);
int c3cu_nccl_unique_id(void* id_out /* 128 bytes */);
int c3cu_nccl_comm_init(void** comm_out, const void* id, int world, int rank);
int c3cu_nccl_comm_destroy(void* comm);
int c3cu_allreduce_grads(void* grads, int64_t count, int dtype, void* comm, c3cu_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* C3CU_H_ */
