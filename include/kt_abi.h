/*
 * kt_abi.h — C ABI of the B200 (sm_100a) tuned-kernel library `libkt.so`.
 *
 * The reference tuner has no library boundary: it writes one `.cu` file per
 * variant whose own `main()` allocates, fills, launches and times the kernel,
 * and Python talks to it through a process + stdout text protocol
 * (`SAMPLE <tag> <ms>`, `TIMING …`, `VERIFY_OUTPUT <v>`;
 * src/generator.py:218-281, src/benchmark.py:157-187, src/verifier.py:531-540).
 * This header replaces that protocol with in-process calls. Every built
 * library — the default `libkt.so` and each generated tuning variant — exports
 * exactly these symbols, so one ctypes (or cgo/JNI) binding serves all of them.
 *
 * Conventions
 *   - Every entry point returns an int status: KT_OK (0) or a KT_ERR_* code.
 *     Nothing here calls exit(), abort() or __trap(); a failure is reported
 *     through the status and kt_last_error() (thread-local text).
 *   - All tensor pointers are CALLER-OWNED device pointers (the reference's
 *     executables allocated their own buffers, src/generator.py:231-249).
 *     The library never frees caller memory.
 *   - `stream` is a cudaStream_t (NULL = legacy default stream). Calls are
 *     asynchronous with respect to the host unless stated otherwise.
 *   - Sizes are int64_t element counts; row-major, densely packed.
 *   - bf16 tensors are passed as uint16_t* holding the raw bf16 bit patterns.
 */
#ifndef KT_ABI_H
#define KT_ABI_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* kt_stream_t; /* identical to cudaStream_t */

/* Libraries are built with hidden visibility; only these entry points are exported. */
#if defined(__GNUC__)
#define KT_API __attribute__((visibility("default")))
#else
#define KT_API
#endif

/* Status codes. The reference mapped every failure (CUDA_CHECK → exit(1),
 * non-zero return, timeout) to `None` in Python (src/benchmark.py:135-152). */
enum {
  KT_OK = 0,
  KT_ERR_ARG = 1,          /* bad pointer / shape / argument                   */
  KT_ERR_CUDA = 2,         /* a CUDA runtime call or a launch failed           */
  KT_ERR_TIMEOUT = 3,      /* a device-side bounded wait gave up               */
  KT_ERR_UNSUPPORTED = 4   /* shape or option this build does not implement    */
};

/* GEMM variants for kt_gemm_f32 (`variant`). */
enum {
  KT_GEMM_FFMA = 0,        /* exact fp32 SIMT FMA path                          */
  KT_GEMM_TF32 = 1         /* tcgen05.mma kind::tf32, fp32 accumulate in TMEM   */
};

/* Operation ids for kt_run / kt_time. */
enum {
  KT_OP_SOFTMAX = 1,
  KT_OP_LAYERNORM = 2,
  KT_OP_REDUCE = 3,
  KT_OP_GEMM = 4,
  KT_OP_FA_FWD = 5,
  KT_OP_NAIVE_SOFTMAX = 101,
  KT_OP_NAIVE_LAYERNORM = 102,
  KT_OP_NAIVE_REDUCE = 103,
  KT_OP_NAIVE_GEMM = 104,
  KT_OP_NAIVE_ATTENTION = 105
};

/* Generic argument block for kt_run / kt_time. Field meaning per op:
 *   SOFTMAX    in0=x           out0=y         d0=rows d1=cols
 *   LAYERNORM  in0=x in1=gamma in2=beta out0=y d0=rows d1=cols f0=eps
 *   REDUCE     in0=x           out0=double*   out1=float* (may be NULL)
 *              workspace/ws_bytes             d0=n
 *   GEMM       in0=A in1=B     out0=C         d0=M d1=N d2=K i0=transpose_b i1=variant
 *   FA_FWD     in0=Q in1=K in2=V out0=O       d0=B d1=H d2=S d3=D f0=scale i0=causal
 *   NAIVE_*    same fields as the matching op (NAIVE_ATTENTION as FA_FWD).   */
typedef struct kt_args {
  const void* in0;
  const void* in1;
  const void* in2;
  void* out0;
  void* out1;
  void* workspace;
  size_t ws_bytes;
  int64_t d0, d1, d2, d3;
  float f0;
  int32_t i0, i1;
} kt_args;

/* Thread-local text of the last error raised on the calling thread ("" if none). */
KT_API const char* kt_last_error(void);

/* ABI version (bumped on any signature change). */
KT_API int kt_version(void);

/* JSON object with the template parameters baked into this build
 * (the reference recorded them only in the generated file's header comment,
 * src/generator.py:29-33). */
KT_API const char* kt_variant_params(void);

/* Row softmax y[r,:] = exp(x[r,:]-max)/sum, fp32 in/out, rows×cols row-major.
 * Replaces `softmax_opt(const float* in, float* out, int rows, int cols)`
 * (src/generator.py:110-153) and `softmax_naive` (src/kernels/baseline_kernels.cu:52-77). */
KT_API int kt_softmax_f32(const float* x, float* y, int64_t rows, int64_t cols, kt_stream_t stream);

/* LayerNorm over the last dim: y = gamma*(x-mean)/sqrt(var+eps)+beta, biased var.
 * Replaces `layernorm_opt(in, out, gamma, beta, rows, cols, eps)`
 * (src/generator.py:166-213) and `layernorm_naive` (src/kernels/baseline_kernels.cu:110-142). */
KT_API int kt_layernorm_f32(const float* x, const float* gamma, const float* beta, float* y,
                     int64_t rows, int64_t cols, float eps, kt_stream_t stream);

/* Bytes of device scratch kt_reduce_sum_f32 needs for n elements. */
KT_API size_t kt_reduce_workspace_bytes(int64_t n);

/* Full sum of n fp32 values, accumulated in fp64; writes *out64 (device) and,
 * when out32 != NULL, the fp32-rounded sum to *out32 (device). `workspace`
 * (>= kt_reduce_workspace_bytes(n) bytes, any content) is caller-owned scratch.
 * Replaces `reduction_opt(const float* in, float* out, int N)`, which only
 * produced per-block partials (src/generator.py:82-98, :302-324), and
 * `reduction_naive` (src/kernels/baseline_kernels.cu:83-104). */
KT_API int kt_reduce_sum_f32(const float* x, int64_t n, double* out64, float* out32,
                      void* workspace, size_t ws_bytes, kt_stream_t stream);

/* Whole-job sum over `world` GPUs, one process per GPU, each holding one
 * contiguous shard of the input: every rank calls this once per step with its
 * shard and gets the sum of all shards (fp64, identical bits on every rank) in
 * *out64 (and *out32 if not NULL). The combine runs inside the kernel: the last
 * CTA of each rank stores its fp64 shard sum into every rank's exchange buffer
 * over NVLink (plain peer stores) and adds the `world` values in rank order
 * once all have arrived. No collective library is called. The wait for the
 * other ranks is bounded (2 s); when it runs out *out64 is NaN and
 * kt_device_error reports 3.
 *   workspace  as kt_reduce_sum_f32 (>= kt_reduce_workspace_bytes(n)), but its
 *              first 4 bytes must be zero before the first call on it (the
 *              kernel leaves them zero), so no per-call reset is issued.
 *   exchange   host array of `world` device pointers: exchange[r] is rank r's
 *              exchange buffer (KT_XRANK_EXCHANGE_BYTES, zeroed before the first
 *              call, 16-byte aligned) as mapped into this process (CUDA IPC or
 *              any symmetric-memory mapping); may be NULL when world == 1.
 *   epoch      1 for the first call on these buffers, +1 for every later call;
 *              all ranks pass the same value.
 * world <= KT_XRANK_MAX. Replaces the per-GPU partial + ncclAllReduce(sum) of
 * one fp64 that a sharded `reduction_opt` would need; the reference's own
 * kernel (src/generator.py:82-98) runs on one GPU only. */
#define KT_XRANK_MAX 8
#define KT_XRANK_EXCHANGE_BYTES 256
KT_API int kt_reduce_sum_f32_xrank(const float* x, int64_t n, double* out64, float* out32,
                                   void* workspace, size_t ws_bytes, void* const* exchange,
                                   int rank, int world, uint64_t epoch, kt_stream_t stream);

/* Same result as kt_reduce_sum_f32, for callers that cannot allocate device
 * memory (host callbacks and real-time loops where cudaMalloc would block or
 * synchronize, embedders with a fixed memory budget, FFI callers holding only
 * their input/output buffers). It allocates nothing: the scratch is a fixed
 * 16 KiB array (KT_NOALLOC_SCRATCH_BYTES; enough for grids of up to 2046 CTAs)
 * in the library's own device memory, present on every device that uses the
 * library until the process exits; a launch needing more returns
 * KT_ERR_UNSUPPORTED. Each call looks the array's device address up with
 * cudaGetSymbolAddress on the current device; the first call on a device also
 * loads the library's device code there, so make that first call outside any
 * stream capture.
 * All calls on a device share the array: calls that may overlap on the GPU
 * (unordered streams) race; order them on one stream.
 * No counterpart in the reference (its executables allocate their own buffers). */
#define KT_NOALLOC_SCRATCH_BYTES 16384
KT_API int kt_reduce_sum_f32_noalloc(const float* x, int64_t n, double* out64, float* out32, kt_stream_t stream);

/* C = A·B (transpose_b=0, B is K×N) or C = A·Bt^T (transpose_b=1, B holds Bt, N×K),
 * fp32 row-major, fp32 output. variant = KT_GEMM_FFMA | KT_GEMM_TF32.
 * Replaces `matmul_opt(const float* A, const float* B, float* C, int N)` with its
 * `transpose_b` load (src/generator.py:40-70, :286-299) and `matmul_naive`
 * (src/kernels/baseline_kernels.cu:32-46). */
KT_API int kt_gemm_f32(const float* A, const float* B, float* C, int64_t M, int64_t N, int64_t K,
                int transpose_b, int variant, kt_stream_t stream);

/* Flash-attention forward, bf16 Q/K/V/O laid out [B,H,S,D] contiguous, fp32
 * softmax and accumulation, O = softmax(scale·Q·K^T [+causal mask])·V.
 * Replaces `attention_flash` / `attention_tiled(Q,K,V,O,S,D)` (single head, fp32;
 * src/attention.py:210-291, :75-176) and `attention_naive`
 * (src/kernels/baseline_kernels.cu:149-181). */
KT_API int kt_fa_fwd_bf16(const uint16_t* Q, const uint16_t* K, const uint16_t* V, uint16_t* O,
                   int64_t B, int64_t H, int64_t S, int64_t D, float scale, int causal,
                   kt_stream_t stream);

/* Naive GPU baselines (one thread per row / per output element) used as the
 * Welch-t reference point, restating the algorithms of
 * src/kernels/baseline_kernels.cu:32-181 (timed by src/kernels/benchmark_runner.cu:236-359). */
KT_API int kt_naive_softmax_f32(const float* x, float* y, int64_t rows, int64_t cols, kt_stream_t stream);
KT_API int kt_naive_layernorm_f32(const float* x, const float* gamma, const float* beta, float* y,
                           int64_t rows, int64_t cols, float eps, kt_stream_t stream);
KT_API int kt_naive_reduce_sum_f32(const float* x, int64_t n, double* out64, float* out32,
                            void* workspace, size_t ws_bytes, kt_stream_t stream);
KT_API int kt_naive_gemm_f32(const float* A, const float* B, float* C, int64_t M, int64_t N, int64_t K,
                      int transpose_b, kt_stream_t stream);
KT_API int kt_naive_attention_bf16(const uint16_t* Q, const uint16_t* K, const uint16_t* V, uint16_t* O,
                            int64_t B, int64_t H, int64_t S, int64_t D, float scale, int causal,
                            kt_stream_t stream);

/* Dispatch one op by id (see kt_args). */
KT_API int kt_run(int op, const kt_args* args, kt_stream_t stream);

/* In-process timing: `warmup` untimed runs, then `iters` samples, each
 * bracketed by its own CUDA event pair on `stream`; between samples the
 * caller-owned `flush` buffer (flush_bytes, may be 0/NULL) is overwritten so
 * that no sample starts with its inputs in L2. Writes iters floats (ms) to
 * samples_ms (host memory) and synchronizes the stream before returning.
 * Replaces the per-variant `main()` timing loop (src/generator.py:255-271) and
 * `time_kernel` (src/kernels/benchmark_runner.cu:74-104). */
KT_API int kt_time(int op, const kt_args* args, int warmup, int iters, void* flush, size_t flush_bytes,
            float* samples_ms, kt_stream_t stream);

/* Device error word written by kernels whose bounded waits gave up
 * (0 = none). Reading it synchronizes the device. reset != 0 clears it. */
KT_API int kt_device_error(int reset, int* code_out);

#ifdef __cplusplus
}
#endif

#endif /* KT_ABI_H */
