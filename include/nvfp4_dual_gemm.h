/*
 * nvfp4_dual_gemm.h — C ABI of the B200 (sm_100a) NVFP4 dual GEMM
 *
 *     C[m, n] = fp16( silu(sum_k A[m,k] * B1[n,k]) * (sum_k A[m,k] * B2[n,k]) )
 *
 * A, B1, B2 are NVFP4: e2m1 codes packed two per byte along K (element 2i in
 * the low nibble, 2i+1 in the high nibble), K-major, with one fp8-e4m3 scale
 * per 16 consecutive K elements.  The scales are passed in the tcgen05
 * "blocked" layout: rows are grouped in blocks of 128 and K/16 scale columns
 * in groups of 4; each (128-row, 4-column) block is one 512-byte atom, atoms
 * ordered row-block major, and inside an atom the scale of (row r, column c)
 * sits at byte (r % 32) * 16 + ((r % 128) / 32) * 4 + (c % 4).  This is the
 * layout the reference kernel reads (nvfp4_dual_gemm.cu:226-243: atom index
 * rowblock * (K/64) + kblock64, 512 bytes per atom).
 *
 * Buffer sizes the caller provides per batch (L problems of one shape, one
 * after another in memory; L = 1 for a single problem):
 *   A    : M * K/2 bytes        row m at A  + m * K/2
 *   B1,B2: N * K/2 bytes        row n at B1 + n * K/2
 *   SFA  : ceil(M/128) * (K/64) * 512 bytes   (blocked, rows padded to 128)
 *   SFB1, SFB2: ceil(N/128) * (K/64) * 512 bytes
 *   C    : M * N fp16, row-major (row m at C + m * N)
 * Batch l of each tensor starts l times its per-batch size after batch 0:
 * the layout of the reference's [rows, cols, L] tensors, which are
 * [L, rows, cols] tensors viewed through permute(1, 2, 0).  The reference
 * kernel reads batch 0 only (its L dimension is ignored); here every batch
 * is computed, all batches' tiles scheduled in one launch.
 *
 * Preconditions (checked, an error code is returned otherwise):
 *   M >= 0, N >= 0, K >= 0; N % 64 == 0; K % 256 == 0; L >= 1 (L == 1 for
 *   nvfp4_dual_gemm_run_noalloc and the host-buffer entry point);
 *   A, B1, B2, SFA, SFB1, SFB2, C 16-byte aligned.
 * M needs no alignment: rows past M are read as zeros and never written.
 *
 * All pointers are device pointers owned by the caller.  `stream` is a
 * cudaStream_t passed as void* (NULL = legacy default stream).  No entry
 * point calls exit(); failures return a non-zero status and the message is
 * available from nvfp4_dual_gemm_last_error() (thread-local).
 */
#ifndef NVFP4_DUAL_GEMM_H_
#define NVFP4_DUAL_GEMM_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define NVFP4DG_API __attribute__((visibility("default")))
#else
#define NVFP4DG_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define NVFP4DG_OK 0
#define NVFP4DG_ERR_INVALID 1     /* bad shape / null pointer / bad L       */
#define NVFP4DG_ERR_ALIGN 2       /* pointer not 16-byte aligned            */
#define NVFP4DG_ERR_WORKSPACE 3   /* workspace missing or too small         */
#define NVFP4DG_ERR_CUDA 4        /* CUDA runtime / driver call failed      */
#define NVFP4DG_ERR_DEVICE 5      /* a kernel reported a bounded-wait timeout */
#define NVFP4DG_ERR_UNSUPPORTED 6 /* device is not sm_100 or entry missing  */

/* `flags` bits for nvfp4_dual_gemm_run / _run_ws (0 = automatic choice).    */
#define NVFP4DG_FLAG_GRID_MASK 0xFFFu  /* bits 0-11: force the persistent grid */
#define NVFP4DG_FLAG_BN64 (1u << 12)   /* force 64-column tiles per GEMM        */
#define NVFP4DG_FLAG_BN128 (1u << 13)  /* force 128-column tiles per GEMM       */
#define NVFP4DG_FLAG_NO_STREAMK (1u << 14) /* whole tiles only (no K split)     */
#define NVFP4DG_FLAG_SYNC_CHECK (1u << 15) /* synchronize and read the device
                                              error word after the launch       */
#define NVFP4DG_FLAG_FORCE_STREAMK (1u << 17) /* always split the last waves of
                                                 tiles along K (stream-K)      */
#define NVFP4DG_FLAG_PAIR (1u << 18)    /* force 2-SM pair tiles (256 rows)    */
#define NVFP4DG_FLAG_NO_PAIR (1u << 19) /* force single-CTA tiles (128 rows)   */
#define NVFP4DG_FLAG_SPLITK (1u << 20)  /* force cluster split-K: the two CTAs
                                           of a cluster take the two halves of
                                           each tile's K range and exchange
                                           their partial sums through
                                           distributed shared memory; needs
                                           2 x tiles <= SMs and K >= 512     */
#define NVFP4DG_FLAG_NO_SPLITK (1u << 21) /* never use cluster split-K       */
#define NVFP4DG_FLAG_NO_PDL (1u << 22)  /* launch without programmatic
                                           dependent launch (by default the
                                           kernel may start while the previous
                                           grid in the stream finishes, and
                                           waits for it before touching global
                                           memory)                            */
#define NVFP4DG_FLAG_STATIC_WEIGHTS (1u << 24) /* the caller guarantees that
                                              no kernel enqueued before this
                                              call writes B1, B2, SFB1 or
                                              SFB2: the weight copies start
                                              before the programmatic
                                              dependency wait, overlapping
                                              the previous kernel's tail
                                              (decode steps on constant
                                              weights); A, SFA and C still
                                              wait.  No effect with
                                              NVFP4DG_FLAG_NO_PDL. */
#define NVFP4DG_FLAG_NO_MERGED_B (1u << 23) /* copy B1 and B2 tiles with
                                              separate copies (by default one
                                              copy brings both when B2 lies
                                              above B1 at a multiple of 16
                                              bytes)                          */
#define NVFP4DG_FLAG_NO_TMA_STORE (1u << 26) /* whole 2-SM pair tiles of
                                              128 columns store their fp16 C
                                              row by row from each thread
                                              instead of staging it in shared
                                              memory for TMA tensor stores */
#define NVFP4DG_FLAG_TEST_SK_TIMEOUT (1u << 25) /* test hook, never for
                                              production: the owner of each
                                              tile split along K (stream-K)
                                              waits for one contribution more
                                              than exist, with a ~1e6-cycle
                                              limit, so that its bounded wait
                                              runs out and the call reports
                                              NVFP4DG_ERR_DEVICE (with
                                              NVFP4DG_FLAG_SYNC_CHECK) or
                                              nvfp4_dual_gemm_device_status
                                              does; the failure path is
                                              tested without a GPU fault.  A
                                              caller-owned workspace must be
                                              zero-filled again afterwards. */

/*
 * Run the dual GEMM on `stream` using a workspace the library keeps per
 * (device, stream); it is allocated (cudaMalloc) on the first call that needs
 * it and reused afterwards.
 *
 * Replaces the reference's torch-extension entry
 *   torch::Tensor cuda_nvfp4_dual_gemm(A, B1, B2, SFA, SFB1, SFB2, C)
 *   (nvfp4_dual_gemm.cu:381-446, declared submission.py:17-20),
 * which derives M = A.size(0), N = B1.size(0), K = 2 * A.size(1) and launches
 * on the legacy default stream.  Unlike the reference, shapes are not limited
 * to a fixed table, and invalid shapes fail instead of returning C untouched
 * (nvfp4_dual_gemm.cu:443-444).
 */
NVFP4DG_API int nvfp4_dual_gemm_run(const void* A, const void* B1, const void* B2,
                        const void* SFA, const void* SFB1, const void* SFB2,
                        void* C, int M, int N, int K, int L, unsigned flags,
                        void* stream);

/*
 * Bytes of workspace nvfp4_dual_gemm_run_ws needs for this problem and flags
 * on the current device (0 when the chosen schedule splits no tile along K).
 * Has no counterpart in the reference, whose kernel never splits K.
 */
NVFP4DG_API size_t nvfp4_dual_gemm_workspace_size(int M, int N, int K, int L,
                                      unsigned flags);

/*
 * Same as nvfp4_dual_gemm_run with a caller-owned workspace of at least
 * nvfp4_dual_gemm_workspace_size() bytes (256-byte aligned).  The workspace
 * must be zero-filled before its first use; every successful call leaves it
 * ready for the next one.  Calls that overlap on the GPU must not share a
 * workspace.  Same reference interface as nvfp4_dual_gemm_run.
 */
NVFP4DG_API int nvfp4_dual_gemm_run_ws(const void* A, const void* B1, const void* B2,
                           const void* SFA, const void* SFB1, const void* SFB2,
                           void* C, int M, int N, int K, int L, unsigned flags,
                           void* workspace, size_t workspace_bytes,
                           void* stream);

/*
 * The dual GEMM with its result emitted in NVFP4 for the next GEMM of the
 * FFN (the down projection, whose K is this N): each 16-column block of a
 * row of the fp16 result h = fp16(silu(A B1^T) * (A B2^T)) is quantised as
 * nvfp4_quantize_rows quantises fp16 rows — scale = e4m3(amax / 6), codes =
 * e2m1(h / scale), round to nearest even, saturating — so the output equals
 * quantising nvfp4_dual_gemm_run's C bit for bit.  Writes
 *   Cq : M * N/2 bytes, row m at Cq + m * N/2 (element 2i in the low nibble)
 *   SFC: ceil(M/128) * (N/64) * 512 bytes, the blocked layout above with
 *        rows = M, K = N; scales of the padding rows up to a multiple of 128
 *        are written as 0, so every byte of the buffer is written.
 * The fp16 C is never materialised.  Same inputs, preconditions, flags and
 * library-owned workspace as nvfp4_dual_gemm_run; Cq and SFC 16-byte
 * aligned.  The reference writes only the fp16 C (nvfp4_dual_gemm.cu:126-193
 * epilogue); its harness would quantise that C on the host for a following
 * NVFP4 GEMM (submission.py:1154 builds such inputs).
 */
NVFP4DG_API int nvfp4_dual_gemm_run_nvfp4_out(
    const void* A, const void* B1, const void* B2, const void* SFA,
    const void* SFB1, const void* SFB2, void* Cq, void* SFC, int M, int N,
    int K, int L, unsigned flags, void* stream);

/*
 * Grouped dual GEMM (mixture-of-experts FFN): `groups` (1..64) problems that
 * share N and K but have their own row counts, in one launch.  Group g's
 * activations are rows [group_row0[g], group_row0[g] + group_rows[g]) of A,
 * SFA and C (group_row0[g] a multiple of 128; groups in increasing order,
 * each group's rows rounded up to 128 ending before the next group starts;
 * rows between groups are neither read into any output nor written), and its
 * weights are batch g of B1, B2, SFB1, SFB2 (per-batch sizes as at the top of
 * this file).  A / C hold max(group_row0[g] + group_rows[g]) rows, SFA the
 * blocked layout of that many rows.  group_rows / group_row0 are HOST arrays,
 * read during the call.  Groups may be empty.  Schedules: 2-SM pair or
 * single-CTA tiles, whole tiles or stream-K (NVFP4DG_FLAG_SPLITK is
 * rejected); `workspace` as for nvfp4_dual_gemm_run_ws (NULL: the library's
 * own), flags otherwise as for nvfp4_dual_gemm_run.  The
 * reference has no grouped form: its tensors' L dimension is ignored
 * (nvfp4_dual_gemm.cu:381-446).
 */
NVFP4DG_API int nvfp4_dual_gemm_run_grouped(
    const void* A, const void* B1, const void* B2, const void* SFA,
    const void* SFB1, const void* SFB2, void* C, const int* group_rows,
    const int* group_row0, int groups, int N, int K, unsigned flags,
    void* workspace, size_t workspace_bytes, void* stream);

/*
 * Bytes of caller-owned workspace nvfp4_dual_gemm_run_grouped needs for
 * these group row counts (0 when its schedule splits no tile along K).
 * With workspace == NULL, nvfp4_dual_gemm_run_grouped uses the library's
 * per-(device, stream) workspace instead, as nvfp4_dual_gemm_run does.  No
 * counterpart in the reference.
 */
NVFP4DG_API size_t nvfp4_dual_gemm_grouped_workspace_size(
    const int* group_rows, int groups, int N, int K, unsigned flags);

/*
 * Quantise fp32 rows to NVFP4 on the GPU: X is [rows, K] fp32 row-major;
 * writes codes [rows, K/2] (low nibble = even element), the plain scales
 * [rows, K/16] and the blocked scales (ceil(rows/128) * (K/64) * 512 bytes;
 * padding rows are written as zero).  Scale = e4m3(amax/6), round to nearest
 * even, saturating at 448; codes = e2m1(x / scale), round to nearest even,
 * saturating at 6; a block whose scale rounds to 0 gets all-zero codes.
 * `sf_plain` may be NULL.  K % 64 == 0.
 * Produces the `data` tuple fields the reference's harness supplies
 * (submission.py:1154: a/b1/b2, sfa/sfb1/sfb2 and the *_blocked copies).
 */
NVFP4DG_API int nvfp4_quantize(const float* X, int rows, int K, void* codes,
                   void* sf_plain, void* sf_blocked, void* stream);

/* Element types of nvfp4_quantize_rows's input. */
#define NVFP4DG_DTYPE_F32 0
#define NVFP4DG_DTYPE_F16 1
#define NVFP4DG_DTYPE_BF16 2

/*
 * Activation quantiser (the step before the dual GEMM in an FFN): X is
 * [rows, K] of `dtype` with a row pitch of `ldx` elements (>= K); writes the
 * e2m1 codes [rows, K/2], the blocked scales (ceil(rows/128) * (K/64) * 512
 * bytes, padding rows zero — every byte of the buffer is written) and, when
 * `sf_plain` is not NULL, the plain scales [rows, K/16].  Same arithmetic
 * as nvfp4_quantize.  K % 64 == 0; X, its row pitch, codes and sf_blocked
 * 16-byte aligned, sf_plain 4-byte aligned.  The reference has no device
 * quantiser: its harness quantises on the host (submission.py:1154).
 */
NVFP4DG_API int nvfp4_quantize_rows(const void* X, int dtype, int rows, int K,
                                    long long ldx, void* codes,
                                    void* sf_plain, void* sf_blocked,
                                    void* stream);

/*
 * Scale layout conversion on the device between the plain layout
 * [rows, K/16] (row pitch `ld` bytes >= K/16) and the blocked layout
 * described at the top of this file (ceil(rows/128) * (K/64) * 512 bytes).
 * to_blocked writes every byte of the blocked buffer (padding rows zero);
 * from_blocked writes the rows x K/16 plain bytes.  K % 64 == 0; plain
 * scales and `ld` 4-byte aligned, blocked scales 16-byte aligned.  The
 * reference's harness builds the blocked copies on the host
 * (submission.py:1154, the `*_blocked` fields of `data`).
 */
NVFP4DG_API int nvfp4_scales_to_blocked(const void* plain, int rows, int K,
                                        long long ld, void* blocked,
                                        void* stream);
NVFP4DG_API int nvfp4_scales_from_blocked(const void* blocked, int rows, int K,
                                          void* plain, long long ld,
                                          void* stream);

/*
 * Read and clear the device error word of `device` (synchronizes that
 * device).  *word_out = 0 when no kernel reported a timeout; otherwise bits
 * identify the role whose bounded wait expired.  Returns a status code.
 */
NVFP4DG_API int nvfp4_dual_gemm_device_status(int device, unsigned* word_out);

/*
 * Describe the schedule the library would use: writes the tile width per
 * GEMM, the CTAs per work unit (1, or 2 for 2-SM pair tiles of 256 rows),
 * the persistent grid in work units, the whole-tile count, the number of
 * tiles split along K by stream-K, and *split_out = 2 when each tile's K
 * range is split between the two CTAs of a cluster (cluster split-K; the
 * grid then counts CTAs, two per tile), else 0.  Any out pointer may be
 * NULL.  Host-only; usable without a GPU when `num_sms` > 0.
 */
NVFP4DG_API int nvfp4_dual_gemm_plan(int M, int N, int K, unsigned flags, int num_sms,
                         int* bn_out, int* ctas_out, int* grid_out,
                         int* dp_tiles_out, int* sk_tiles_out,
                         int* split_out);

/*
 * Enumerate the work of work unit `cta` (a CTA, or a CTA pair) under the plan
 * for (M, N, K, flags, num_sms): writes up to `cap` records of 4 ints (tile,
 * kb_begin, kb_end, slot; slot = -1 for a whole tile) and returns the record
 * count, or -1 on error.  Host-only mirror of the device scheduler, for tests
 * and tooling.
 */
NVFP4DG_API int nvfp4_dual_gemm_plan_work(int M, int N, int K, unsigned flags, int num_sms,
                              int cta, int* records, int cap);

/*
 * Upper limit, in bytes, of the scratch buffer nvfp4_dual_gemm_run_noalloc
 * keeps in device memory.
 */
#define NVFP4DG_NOALLOC_SCRATCH_BYTES (4u << 20)

/*
 * Same computation as nvfp4_dual_gemm_run, for callers that cannot allocate
 * device memory at the time they call: code running where cudaMalloc is not
 * allowed or not wanted (inside a custom memory arena or pool that owns all
 * device memory, a framework whose allocator must not be re-entered, a
 * real-time path that must not block on the allocator).  No counterpart in
 * the reference: its kernel never needs scratch memory.
 *
 * Tiles split along K need fp32 scratch; this entry point takes it from a
 * static array of NVFP4DG_NOALLOC_SCRATCH_BYTES that every GPU which loads
 * the library holds until the process exits, and it calls no cudaMalloc,
 * cudaFree or other allocating routine.  The caller passes inputs and
 * outputs as for nvfp4_dual_gemm_run, for one problem: L must be 1 (batched
 * problems go through nvfp4_dual_gemm_run or nvfp4_dual_gemm_run_ws).  The
 * first call on a device looks up the array's device address
 * (cudaGetSymbolAddress) with that device current; make that first call
 * before any stream capture.  When the automatic schedule would need more
 * scratch than the array holds, the call runs whole tiles instead (no
 * scratch); only a schedule forced with NVFP4DG_FLAG_FORCE_STREAMK that
 * does not fit is rejected with NVFP4DG_ERR_WORKSPACE
 * (nvfp4_dual_gemm_run_ws takes a larger caller-owned buffer).
 * Every call shares the one array, which keeps the last call's contents:
 * each call clears the tile counters it needs before launching.  Each
 * device has its own copy of the array, but calls that overlap on the GPU of
 * one device (for example on two streams) race on it and must be serialised
 * by the caller.
 */
NVFP4DG_API int nvfp4_dual_gemm_run_noalloc(
    const void* A, const void* B1, const void* B2, const void* SFA,
    const void* SFB1, const void* SFB2, void* C, int M, int N, int K, int L,
    unsigned flags, void* stream);

/*
 * Host-buffer entry point: A, B1, B2, SFA, SFB1, SFB2 and C are HOST buffers
 * (page-locked for the copies to overlap; any alignment), with the sizes and
 * layouts listed at the top of this file.  The library uploads the inputs
 * into `staging`, a caller-owned device buffer of at least
 * nvfp4_dual_gemm_host_staging_size(M, N, K, L) bytes (256-byte aligned),
 * computes, and downloads C.  The weights go up in slabs of whole 128-row
 * groups of B1/B2; each slab's kernel starts as soon as its slab has landed
 * and each slab of C goes back while later slabs still go up, so the two
 * directions of the host link and the kernels overlap.  Each copy costs a
 * few microseconds beyond its bytes, so more slabs pay only when the
 * download is long enough to hide behind the upload: `slabs` = 0 picks the
 * count (1 to 16) from a model of the link; 1 runs upload, kernel and
 * download back to back.  The copies run on two streams of the library's
 * own, ordered after the work already queued on `stream`; `stream` waits for
 * them, so host C is complete once `stream` is.  Calls on one `stream` may
 * share a staging buffer.
 *
 * Replaces the reference's `custom_kernel(data)` (submission.py:1153-1157)
 * for a caller whose tensors are in host memory: the reference's entry
 * takes device tensors only (nvfp4_dual_gemm.cu:381-446), so such a caller
 * copies every input up, calls it and copies C back, one after another.
 */
NVFP4DG_API size_t nvfp4_dual_gemm_host_staging_size(int M, int N, int K, int L);

/* Slab count nvfp4_dual_gemm_run_host uses for M, N, K and a requested
 * count (0 = automatic); 0 for invalid arguments.  Host-only. */
NVFP4DG_API int nvfp4_dual_gemm_host_slabs(int M, int N, int K, int slabs);

NVFP4DG_API int nvfp4_dual_gemm_run_host(
    const void* A, const void* B1, const void* B2, const void* SFA,
    const void* SFB1, const void* SFB2, void* C, int M, int N, int K, int L,
    unsigned flags, int slabs, void* staging, size_t staging_bytes,
    void* stream);

/* Thread-local message describing the last failure ("" if none). */
NVFP4DG_API const char* nvfp4_dual_gemm_last_error(void);

/* ABI version: major * 100 + minor. */
NVFP4DG_API int nvfp4_dual_gemm_version(void);

#ifdef __cplusplus
}
#endif

#endif /* NVFP4_DUAL_GEMM_H_ */
