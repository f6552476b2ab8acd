/*
 * kl_gemm.h — C ABI of the B200 dense-GEMM engine (libkl_b200.so).
 *
 * Plain pointers, sizes and status codes only, so any FFI (ctypes, cgo, JNI, N-API) can bind it.
 * The reference (govindansriram/maia, kernel_lib) is a header-only C++20 library with no C ABI;
 * each entry point below names the reference interface it exposes (file:line inside the
 * reference project) or says that it has none.
 *
 * Memory: every pointer named "device" is CUDA device memory owned by the caller; the library
 * keeps no pointer after a call returns. `stream` is a cudaStream_t (NULL = legacy default
 * stream). GEMM launches are stream-ordered and asynchronous: they return once the kernel is
 * queued. No entry point throws; failures return a kl_status and kl_last_error() describes the
 * latest failure on the calling thread.
 */
#ifndef KL_GEMM_H_
#define KL_GEMM_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define KL_API __attribute__((visibility("default")))
#else
#define KL_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum kl_status {
  KL_OK = 0,
  KL_ERR_INVALID_ARGUMENT = 1, /* bad shape, stride, alignment or combination */
  KL_ERR_NOT_SUPPORTED = 2,    /* a valid request this library or device cannot run */
  KL_ERR_CUDA = 3,             /* a CUDA runtime/driver call failed */
  KL_ERR_TIMEOUT = 4,          /* a bounded device-side wait ran out (kl_read_status) */
  KL_ERR_NCCL = 5              /* reserved for collective failures */
} kl_status;

typedef enum kl_dtype {
  KL_BF16 = 0,
  KL_F16 = 1,
  KL_E4M3 = 2,
  KL_E5M2 = 3,
  KL_F32 = 4,
  KL_I8 = 5,
  KL_U8 = 6,
  KL_I32 = 7,
  KL_E2M1 = 8,  /* fp4, two per byte (first in the low nibble); extents and pitches count elements */
  KL_UE8M0 = 9, /* block-scale formats */
  KL_UE4M3 = 10,
  KL_E3M2 = 11, /* fp6, packed: element i of a row at bits [6i, 6i + 6) of its bytes (four in three);
                 * extents and pitches count elements */
  KL_E2M3 = 12
} kl_dtype;

typedef enum kl_algo {
  KL_ALGO_AUTO = 0,
  KL_ALGO_1CTA = 1,   /* 128 x 256 tile per CTA, cta_group::1 */
  KL_ALGO_2CTA = 2,   /* 256 x 256 tile per CTA pair, cta_group::2 */
  KL_ALGO_SKINNY = 3  /* memory-bound small-M path: weights stream once, K split over all SMs */
} kl_algo;

/* C[M,N] = alpha * (A[M,K] . B[N,K]^T) [* *scale_a * *scale_b].
 * A and B are K-major (row-major with K contiguous), C is row-major. Leading dimensions are in
 * elements; every base address must be 16-byte aligned and every row pitch a multiple of 16 bytes
 * (TMA rules). */
typedef struct kl_gemm_desc {
  int64_t m, n, k;
  const void* a; /* device, [m, lda] */
  int64_t lda;
  const void* b; /* device, [n, ldb] */
  int64_t ldb;
  void* c;       /* device, [m, ldc] */
  int64_t ldc;
  int32_t ab_type;        /* kl_dtype of A and B: KL_BF16, KL_F16, KL_E4M3, KL_E5M2, KL_E2M1
                             (packed fp4, block-scaled only) or KL_E3M2 / KL_E2M3 (packed fp6,
                             block_scale = 1 only) */
  int32_t c_type;         /* kl_dtype of C. (ab_type, c_type): (bf16, bf16), (bf16, f32), (f16, f16),
                             (f16, f32), (e4m3, bf16), (e4m3, f32), (e5m2, bf16), (e5m2, f32).
                             KL_ALGO_SKINNY: (bf16, bf16), (bf16, f32), (e4m3, bf16) */
  float alpha;            /* host scalar */
  const float* scale_a;   /* optional device scalar (NULL = 1): per-tensor dequant scale of A */
  const float* scale_b;   /* optional device scalar (NULL = 1) */
  int32_t algo;           /* kl_algo */
  int32_t group_m;        /* tile-raster group height in tiles; 0 = library default */
  int32_t max_ctas;       /* cap on resident CTAs; 0 = one per SM */
  int32_t variant;        /* algorithm variant, 0 = library default. KL_ALGO_SKINNY: weight rows
                             per tile / 128 (1 or 2). KL_ALGO_2CTA without block scaling: 1 = 256 x 256
                             tiles, 4 = 256 x 512 tiles (two MMAs of N = 256 per stage of A; (bf16,
                             bf16) and (e4m3, bf16), K-major, 128-byte swizzle, no split tail), 0 =
                             256 x 512 for bf16 where they fill as many worker-waves as 256 x 256
                             tiles and those need no split tail (8192^3, N-shards of 1024), else
                             256 x 256 */
  int32_t prefetch;       /* L2 prefetch distance in K-blocks: 0 = library default, < 0 = off */
  /* Batched GEMM: `batch` independent problems (0 or 1 = one), matrix i of A/B/C at
   * a/b/c + i * stride_a/b/c elements (strides positive, multiples of 16 bytes). Tile kernels
   * only (KL_ALGO_AUTO picks one). */
  int64_t batch;
  int64_t stride_a, stride_b, stride_c;
  /* Operand storage: 0 = K-major (A [M, K], B [N, K], K contiguous), 1 = MN-major (A stored
   * [K, M] with M contiguous, B stored [K, N]); lda / ldb are then the pitch of the stored
   * matrix. MN-major operands: bf16 inputs with bf16 C on the tile kernels. */
  int32_t a_major, b_major;
  /* 0: C = result. 1 (add): C += result (split-K partial sums, a residual add). fp32 C: the tile
   * kernels add with TMA reducing stores (cp.reduce.async.bulk.tensor .add, performed by the TMA
   * unit). bf16 / f16 C: the epilogue reads C, adds in fp32 and stores the sum, rounded once. The
   * skinny kernel: a read-modify-write by the one thread that owns each element. Calls that add
   * into one C from the same stream are ordered; concurrent calls race. */
  int32_t c_reduce;
  /* Operand swizzle span in bytes: 0 (= 128), 128, 64 or 32. 64 and 32 select tile kernels whose
   * stages hold the same 128 bytes of K as two or four swizzle atoms (one TMA box each); bf16
   * inputs with bf16 or f32 C, K-major operands. */
  int32_t swizzle;
  /* Block scaling. 2 (NVFP4): ab_type KL_E2M1 with one UE4M3 scale (an e4m3 value, sign 0) per 16
   * K-elements, blocked by kl_pack_block_scales(vec 16); otherwise as for 1.
   * 0: none. 1 (MX): ab_type KL_E4M3, KL_E5M2, KL_E2M1, KL_E3M2 or KL_E2M3 with one UE8M0 scale (value
   * 2^(s - 127)) per 32 consecutive K-elements of every row of A and of B, in `sfa` / `sfb`
   * (device), stored in the 128 x 4 blocked layout that kl_mx_pack_scales writes:
   * kl_mx_scale_bytes(rows, k) bytes. C = alpha * sum_k (A[m,k] sfa[m,k/32]) (B[n,k] sfb[n,k/32])
   * [* *scale_a * *scale_b]; C bf16 or f32 (KL_ALGO_2CTA: variant 0/1 = 256 x 256 tiles on a CTA
   * pair, 2 = 256 x 128, 3 = 256 x 192; KL_ALGO_1CTA: variant 0/1 = 128 x 256, 2 = 128 x 128;
   * KL_ALGO_SKINNY: up to 128 rows of A, bf16 C, e4m3, e3m2, e2m3 or e2m1; KL_ALGO_AUTO: skinny up to 128 rows,
   * the pair from 256), K-major operands, 128-byte swizzle, batch 1. fp6 (KL_E3M2 / KL_E2M3): K,
   * lda, ldb and stride_b multiples of 128 elements (96 bytes), A and B 32-byte aligned. */
  int32_t block_scale;
  /* Tile kernels (KL_ALGO_1CTA / 2CTA, and AUTO's choice of them): 0 = where dealing whole tiles
   * leaves the last wave short (N-sharded GEMMs: 128 tiles of 256 x 256 on 74 CTA pairs), cut each
   * tile of that wave into 2-4 K-ranges spread over every worker; 1 = always cut the last wave; -1 =
   * never. The ranges are summed through a per-stream library workspace (78 MiB, allocated on first
   * use, never inside a stream capture: a capture that finds none runs whole tiles) in range order:
   * results are deterministic but can differ in the last bits from whole-tile results. */
  int32_t stream_k;
  const void* sfa;
  const void* sfb;
  /* m-grouped GEMM (mixture-of-experts layout): m_block_group non-NULL makes B a stack of `groups`
   * matrices [groups, N, K] (stride_b elements apart) while A [M, K] and C [M, N] stay single
   * matrices whose rows are the groups' rows back to back, each group padded to a multiple of 128
   * rows. m_block_group (device, ceil(M / 128) int32) names the B of every 128-row block; -1 marks
   * a padding block (its C rows come out 0, or C + 0). KL_ALGO_AUTO / KL_ALGO_1CTA: the one-CTA
   * tile kernel, any such layout; KL_ALGO_2CTA: the CTA pair, which takes each 256-row tile's
   * group from its first block, so groups must be padded to 256 rows (blocks 2i and 2i + 1 name the
   * same group). K-major, batch 1. With block scaling, sfb holds the groups' blocked scale arrays
   * back to back (kl_block_scale_bytes(N, K, vec) bytes each) and sfa A's. */
  int32_t groups;
  /* Programmatic dependent launch (tile and skinny kernels): 0 = library default (on), 1 = on,
   * -1 = off. On, the launch may start while the kernel before it on the stream is finishing: its
   * CTAs set up shared memory, barriers and TMEM on SMs that kernel has left, and wait for it to
   * complete (its writes visible) before reading or writing any global memory. Results and
   * stream order are those of a plain launch. */
  int32_t launch_overlap;
  const int32_t* m_block_group;
} kl_gemm_desc;

/* ---- block scale factors (MX, NVFP4) ------------------------------------------------------
 * The blocked layout: rows in blocks of 128, K in blocks of 4 scales (4 * vec elements); each
 * (row block, K block) is a 512-byte atom, atoms stored row-block major ((rb * kb_count + kb) *
 * 512), and inside an atom the scale of row r, K-group j sits at byte (r % 32) * 16 + (r / 32) * 4
 * + j. Padding rows and K-groups hold a scale of 1. No counterpart in the reference. */

/* Bytes of the blocked scale array for `rows` rows and `k` K-elements, one scale per `vec` (32 for
 * MX, 16 for NVFP4) elements: ceil(rows / 128) * ceil(k / (4 * vec)) * 512. */
KL_API int64_t kl_block_scale_bytes(int64_t rows, int64_t k, int32_t vec);
KL_API int64_t kl_mx_scale_bytes(int64_t rows, int64_t k); /* vec = 32 */

/* Device: repack row-major scales src[rows][ceil(k / vec)] (one byte each, row pitch ld_src
 * bytes) into the blocked layout at dst (kl_block_scale_bytes bytes, 16-byte aligned); padding
 * holds a scale of 1 (UE8M0 127 for vec 32, UE4M3 0x38 for vec 16). Stream-ordered. */
KL_API kl_status kl_pack_block_scales(const void* src, int64_t rows, int64_t k, int32_t vec, int64_t ld_src,
                                      void* dst, void* stream);
KL_API kl_status kl_mx_pack_scales(const void* src, int64_t rows, int64_t k, int64_t ld_src, void* dst,
                                   void* stream); /* vec = 32 */

/* Device: MX quantisation (OCP Microscaling Formats v1.0) of x [rows, k] (KL_F32 or KL_BF16, row
 * pitch ldx elements; k a multiple of 32) into q (KL_E4M3: [rows, ldq] bytes; KL_E2M1: packed,
 * ldq elements = ldq / 2 bytes per row; KL_E3M2 / KL_E2M3: packed fp6, ldq a multiple of 128
 * elements = 3 ldq / 4 bytes per row) and the blocked UE8M0 scales (kl_block_scale_bytes(rows, k,
 * 32) bytes, padding included): per 32 elements, scale 2^(floor(log2(amax)) - emax) with emax 8
 * (e4m3), 4 (e3m2) or 2 (e2m1, e2m3), elements x / scale rounded to nearest even, saturating.
 * Stream-ordered; the outputs feed kl_gemm with block_scale = 1 directly. */
KL_API kl_status kl_mx_quantize(const void* x, int32_t x_type, int64_t rows, int64_t k, int64_t ldx, int32_t q_type,
                                void* q, int64_t ldq, void* scales, void* stream);

/* Device: NVFP4 quantisation of x [rows, k] (KL_F32 or KL_BF16, row pitch ldx elements; k a
 * multiple of 16): a per-tensor scale g = amax(|x|) / (448 * 6) (1 for an all-zero x), written as
 * fp32 to *global_scale (device); per 16 consecutive elements a UE4M3 scale s = e4m3(amax_16 /
 * (6 g)) (nearest, saturating) into `scales` in the blocked layout (kl_block_scale_bytes(rows, k,
 * 16) bytes, padding 0x38 = 1.0); elements e2m1(x / (s g)) packed two per byte into q (ldq
 * elements per row, a multiple of 32). x ~ g * s * q. All arithmetic in fp64, so the result
 * equals a host restatement bit for bit. Three kernels on `stream`; the outputs feed kl_gemm with
 * block_scale = 2 (scale_a / scale_b = the global scales). */
KL_API kl_status kl_nv_quantize(const void* x, int32_t x_type, int64_t rows, int64_t k, int64_t ldx, void* q,
                                int64_t ldq, void* scales, float* global_scale, void* stream);

/* Frees every workspace the library allocated for kl_gemm (the skinny kernel's per-device buffer,
 * the tile kernels' per-stream split-tail buffers), after synchronising each device that has one;
 * later calls allocate afresh. No launch that uses them may be in flight or captured in a CUDA
 * graph that will still be replayed. KL_OK when there is nothing to free. It also forgets the
 * cached device address of kl_gemm_skinny_noalloc's scratch array: call it after resetting a device
 * (cudaDeviceReset) and before the next kl_gemm_skinny_noalloc call on that device. */
KL_API kl_status kl_release_workspaces(void);

/* Library version: major * 10000 + minor * 100 + patch. */
KL_API int32_t kl_version(void);

/* Message of the latest failure on this thread ("" if none). */
KL_API const char* kl_last_error(void);

/* No reference counterpart: kernel_lib has descriptor builders only (layout/tma_desc.hpp,
 * layout/umma_desc.hpp) and no GEMM. Queues one GEMM on `stream`. */
KL_API kl_status kl_gemm(const kl_gemm_desc* desc, void* stream);

/* No reference counterpart. Bytes of device workspace kl_gemm needs for `desc` (0 for every
 * algorithm except KL_ALGO_SKINNY, which keeps fp32 partial sums). */
KL_API kl_status kl_gemm_workspace_size(const kl_gemm_desc* desc, size_t* bytes);

/* No reference counterpart. The kernel family kl_gemm runs for `desc` (KL_ALGO_1CTA, KL_ALGO_2CTA
 * or KL_ALGO_SKINNY): desc->algo, or the library's choice for KL_ALGO_AUTO. Reads only the
 * descriptor's extents, types and options; launches nothing and needs no GPU. */
KL_API kl_status kl_gemm_resolve_algo(const kl_gemm_desc* desc, int32_t* algo);

/* No reference counterpart. The C tile (rows x columns) of the kernel kl_gemm runs for `desc`:
 * 128 x 256 (or 128 x 128) on one CTA, 256 x 256, 256 x 512, 256 x 192 or 256 x 128 on a CTA pair,
 * 0 x 0 for the stream-K skinny kernel. The CTA-pair choice of variant 0 depends on the current
 * device's SM count, so this needs a CUDA device (KL_ERR_CUDA without one); nothing is launched. */
KL_API kl_status kl_gemm_resolve_tile(const kl_gemm_desc* desc, int32_t* tile_m, int32_t* tile_n);

/* No reference counterpart. Like kl_gemm, with caller-provided device workspace: at least
 * kl_gemm_workspace_size bytes, 16-byte aligned, zero-filled before its first use. Its head holds
 * 16 bytes of arrival counters per 128 rows of B, which the skinny kernel leaves at zero after
 * every call; the partial sums after them are overwritten each call. So the buffer can be reused
 * as is for any call whose B has at most as many rows as the previous call's; before a call with
 * more rows of B, zero it again (or just its first 16 * ceil(N / 128) bytes). Calls that share one
 * workspace must not overlap on the GPU. After kl_read_status reports KL_ERR_TIMEOUT, zero it
 * again. (kl_gemm without a workspace uses one library-owned buffer per device, with the same
 * no-overlap rule, and does all of this itself.) */
KL_API kl_status kl_gemm_ws(const kl_gemm_desc* desc, void* workspace, size_t workspace_bytes, void* stream);

/* No reference counterpart. The same GEMM with A, B and C in HOST memory (page-locked for full
 * speed): desc->a, desc->b, desc->c are host pointers with desc's leading dimensions, and dev_a,
 * dev_b, dev_c are device buffers of at least m*lda, n*ldb, m*ldc elements that the call uses as
 * staging. The library copies A in, then streams B in `chunks` column blocks of C (0 = choose; a
 * block is a multiple of 256 columns) so that the copy in of block j+1, the GEMM of block j and
 * the copy back of block j-1 overlap. Ordered after the work already on `stream`; `stream` waits
 * for C to be on the host. The call only queues work: synchronise `stream` before reading C.
 * Block scaling (block_scale 1 or 2): desc->sfa / desc->sfb are HOST pointers to the blocked scale arrays;
 * the library stages them in a device buffer of its own (one per device, grown on demand). K-major
 * operands, C output only (c_reduce 0), one problem per call. */
KL_API kl_status kl_gemm_host(const kl_gemm_desc* desc, void* dev_a, void* dev_b, void* dev_c, int32_t chunks,
                              void* stream);

/* No reference counterpart. kl_gemm_host with A already in device memory: desc->a (and desc->sfa
 * when block-scaled) are DEVICE pointers, desc->b, desc->c (and desc->sfb) host pointers staged
 * through dev_b / dev_c as in kl_gemm_host. The copies of B start once the work already on `stream`
 * is done; the GEMMs also wait for `a_ready` (a cudaEvent_t the caller recorded after whatever
 * produces A, e.g. an all-gather of A's row slabs from the other GPUs; NULL = none). This is the
 * per-GPU half of an end-to-end N-sharded GEMM in which each GPU copies only its slab of A over
 * PCIe. */
KL_API kl_status kl_gemm_host_b(const kl_gemm_desc* desc, void* a_ready, void* dev_b, void* dev_c, int32_t chunks,
                                void* stream);

/* No counterpart in the reference. The skinny (KL_ALGO_SKINNY) GEMM for callers that may not
 * allocate device memory while they run and cannot lend the library a workspace (for example an
 * inference-runtime plugin that is handed only its input and output tensors, or a serving loop
 * that forbids allocation after warm-up). Its scratch is a fixed 16 MiB array inside the library,
 * reserved on every GPU that loads it for the life of the process; this call allocates nothing.
 * Limits: at most 256 rows of A, at most 524288 rows of B, and (ceil(N/128) + SMs - 1) x
 * token_tile x 512 bytes of partial sums within 16 MiB - 64 KiB (token_tile = M rounded up to 16,
 * 32, 64, 128 or 256; at N = 28672 on a 148-SM B200 that is M <= 64); larger problems are
 * rejected with KL_ERR_INVALID_ARGUMENT and a message. The first call on a device looks up the
 * array's device address (cudaGetSymbolAddress); make that first call before any stream capture.
 * Under CUDA's lazy module loading (the default) that first call is also what loads the module
 * holding the array, i.e. where its 16 MiB are committed: make it a warm-up call, made while
 * memory is still free; it can fail with KL_ERR_CUDA (out of memory) where a later one cannot.
 * Every call shares the one array, which keeps the last call's contents: each call clears the
 * arrival counters it uses on `stream` before its kernel, and calls that overlap on the GPU race
 * on the array, so serialise them. desc->algo must be KL_ALGO_AUTO or KL_ALGO_SKINNY;
 * desc->variant 0 or 1 (both the one-box kernel; variant 2 is KL_ERR_NOT_SUPPORTED here); C
 * aligned to its element size. A call that is rejected queues nothing on `stream`. The kernel is
 * launched plainly (desc->launch_overlap is not used): its arrival counters are cleared by a
 * cudaMemsetAsync queued just before it. */
KL_API kl_status kl_gemm_skinny_noalloc(const kl_gemm_desc* desc, void* stream);

/* No reference counterpart. The tile-kernel GEMM (KL_ALGO_1CTA / 2CTA) whose epilogue also writes
 * every finished tile of C into `n_peers` (<= 7) other copies of C: device pointers of the same
 * shape and pitch in other GPUs' memory, mapped into this process (kl_ipc_open_handle). With
 * desc->b one rank's column shard of B and desc->c that shard's columns of the full C on every
 * GPU, the GEMM leaves the whole C on every GPU without a separate all-gather: the NVLink
 * transfers overlap the next tiles' math. The kernel only stores to peer memory. Before reading C,
 * every rank's kernel must have finished (e.g. a stream-ordered collective after this call). */
KL_API kl_status kl_gemm_gather(const kl_gemm_desc* desc, void* const* peer_c, int32_t n_peers, void* stream);

/* No reference counterpart. The same gather through NVLink multicast: `mc_c` is the multicast
 * address of desc->c (the same element and pitch, in a buffer bound to an NVSwitch multicast object
 * on every GPU of the group, e.g. torch's symmetric memory `multicast_ptr` plus desc->c's offset).
 * The epilogue writes every finished tile once with multimem stores, which the switch delivers to
 * every GPU's copy of C, this one's included, so each GPU sends its shard once instead of once per
 * peer. Tile kernels (KL_ALGO_1CTA / 2CTA, AUTO picks), one problem, C = result (c_reduce 0); the
 * base, pitch and width of C multiples of 16 bytes. Before another GPU reads C, this GPU's kernel
 * must have finished and a synchronisation across the GPUs must order that read after it (e.g. a
 * collective queued on `stream` after this call). */
KL_API kl_status kl_gemm_gather_multicast(const kl_gemm_desc* desc, void* mc_c, void* stream);

/* ---- Bounded collectives for the N-sharded path. No counterpart in the reference (it has no
 * multi-GPU code); the failure contract follows its status-code style (tma_desc.hpp:134-152 throws,
 * this ABI returns codes). An NCCL communicator created non-blocking: initialisation, enqueueing
 * and completion are polled against a host deadline, and NCCL's asynchronous errors are read on
 * every poll. When the deadline passes (a rank has left, a link is down) or an error shows, the
 * communicator is aborted, which also ends its kernels still waiting on the GPU, the stream is
 * drained, and the call returns KL_ERR_TIMEOUT or KL_ERR_NCCL instead of hanging; every later use
 * of the communicator returns KL_ERR_NCCL. NCCL is loaded at run time (the libnccl.so.2 already in
 * the process, else the system's); without it these return KL_ERR_NOT_SUPPORTED. */
typedef struct kl_comm kl_comm;
/* 128 bytes that every rank passes to kl_comm_init (made on one rank, sent to the others). */
KL_API kl_status kl_comm_get_unique_id(void* id);
KL_API kl_status kl_comm_init(const void* id, int32_t world, int32_t rank, int64_t timeout_ms, kl_comm** comm);
/* recv (world x bytes) = every rank's `bytes` of send, in rank order; queued on `stream`. */
KL_API kl_status kl_comm_all_gather(kl_comm* comm, const void* send, void* recv, int64_t bytes, void* stream);
/* Waits until `stream` (with the communicator's collectives on it) is done, at most timeout_ms. */
KL_API kl_status kl_comm_wait(kl_comm* comm, void* stream, int64_t timeout_ms);
KL_API int32_t kl_comm_is_aborted(const kl_comm* comm);
/* Finalises (waiting at most timeout_ms for the other ranks) and frees; an aborted one is only freed. */
KL_API kl_status kl_comm_destroy(kl_comm* comm, int64_t timeout_ms);

/* CUDA IPC for peer copies of C: a 64-byte handle of the device allocation that contains dev_ptr
 * plus dev_ptr's byte offset inside it; kl_ipc_open_handle maps the allocation in another process
 * (peer access enabled lazily) and returns its base: add the offset. */
KL_API kl_status kl_ipc_get_handle(const void* dev_ptr, void* handle, int64_t* offset);
KL_API kl_status kl_ipc_open_handle(const void* handle, void** dev_ptr);
KL_API kl_status kl_ipc_close(void* dev_ptr);

/* No reference counterpart; a diagnostic. Runs one tile-kernel GEMM (KL_ALGO_1CTA / 2CTA) with
 * every CTA recording {clock64, %globaltimer} at its start and end, waits for it, and copies the
 * 4 words per CTA to `out` (host, out_words >= 4 * CTAs); *ctas receives the CTA count. The ratio
 * of cycles to nanoseconds is the SM clock the kernel actually ran at. */
KL_API kl_status kl_gemm_clock_probe(const kl_gemm_desc* desc, uint64_t* out, int32_t out_words, int32_t* ctas,
                                     void* stream);

/* Upper bound on any device-side wait, in nanoseconds (default 2e9). A wait that runs out sets a
 * bit in the device status word instead of hanging the GPU. */
KL_API void kl_set_wait_timeout_ns(uint64_t ns);

/* Synchronises the current device, then returns KL_ERR_TIMEOUT if any kernel on it recorded a
 * timed-out wait since the last clear (bits in *bits, may be NULL), else KL_OK. clear != 0 resets. */
KL_API kl_status kl_read_status(int32_t* bits, int32_t clear);

/* Launches a one-thread kernel that waits on an mbarrier nobody arrives on, with `timeout_ns` as
 * its bound: the failure path of every kl wait, exercised without harming the GPU. The kernel
 * records a timeout bit; read it back with kl_read_status. */
KL_API kl_status kl_probe_wait_timeout(uint64_t timeout_ns, void* stream);

/* ---- descriptor encoders (host, no GPU needed except kl_make_tma_desc) ---------------------- */

/* Element offset of (row, col) in a rows x cols shared-memory tile of `elem_bytes`-byte elements,
 * swizzled (`swizzled`) and before the swizzle (`plain`). swizzle_span: 16 (none), 32, 64, 128.
 * kernel_lib/include/kl/layout/smem_tile.hpp:33-42 (smem_atom / smem_layout). */
KL_API kl_status kl_smem_tile_offset(int32_t elem_bytes, int32_t rows, int32_t cols, int32_t swizzle_span, int32_t row,
                              int32_t col, int64_t* swizzled, int64_t* plain);

typedef struct kl_tma_box {
  int32_t inner, outer, col_boxes, row_boxes, count, bytes;
} kl_tma_box;

/* TMA box geometry of a tile, and box i's (row, col, smem byte offset).
 * kernel_lib/include/kl/layout/tma_desc.hpp:47-74 (TmaBox). */
KL_API kl_status kl_tma_box_geometry(int32_t elem_bytes, int32_t rows, int32_t cols, int32_t swizzle_span, kl_tma_box* out);
KL_API kl_status kl_tma_box_position(int32_t elem_bytes, int32_t rows, int32_t cols, int32_t swizzle_span, int32_t box,
                              int32_t* row, int32_t* col, uint32_t* smem_offset);

/* 64-bit UMMA shared-memory descriptor of K-slice `k_block`, rows from `row`, of a K-major tile at
 * shared address `tile_addr`. kernel_lib/include/kl/layout/umma_desc.hpp:19-47
 * (num_k_blocks, block_offset_16B, umma_desc). */
KL_API kl_status kl_umma_smem_desc(int32_t elem_bytes, int32_t rows, int32_t cols, int32_t swizzle_span, uint32_t tile_addr,
                            int32_t k_block, int32_t row, uint64_t* out);

/* 32-bit tcgen05.mma instruction descriptor, both operands K-major. M = 64/128 (one CTA) or 256
 * (CTA pair). kernel_lib/include/kl/layout/umma_desc.hpp:49-58 (mma_instr_desc, M <= 128 there). */
KL_API kl_status kl_mma_instr_desc(int32_t a_type, int32_t b_type, int32_t acc_type, int32_t m, int32_t n, uint32_t* out);

/* 32-bit instruction descriptor of a block-scaled tcgen05.mma: a_type / b_type KL_E4M3, KL_E5M2,
 * KL_E3M2 or KL_E2M3 (kind::mxf8f6f4) or KL_E2M1 (kind::mxf4 / mxf4nvf4), scale_type KL_UE8M0 or KL_UE4M3,
 * M = 128 or 256, K-major operands; a_sf_id / b_sf_id (0-3) select the byte of each TMEM scale
 * word the MMA reads first. No counterpart in the reference; pinned to CuTe's
 * make_instr_desc_block_scaled / make_runtime_instr_desc_block_scaled. */
KL_API kl_status kl_mma_instr_desc_block_scaled(int32_t a_type, int32_t b_type, int32_t scale_type, int32_t m,
                                                int32_t n, int32_t a_sf_id, int32_t b_sf_id, uint32_t* out);

/* MN-major form of kl_umma_smem_desc: a tile stored k_rows x mn_cols (MN contiguous, swizzle
 * 32/64/128 bytes), K-slice `k_block`, MN columns [mn_col, mn_col + mn_extent) (0 = to the end).
 * No counterpart in the reference (K-major only); pinned to CuTe's make_umma_desc<Major::MN>. */
KL_API kl_status kl_umma_smem_desc_mn(int32_t elem_bytes, int32_t k_rows, int32_t mn_cols, int32_t swizzle_span,
                                      uint32_t tile_addr, int32_t k_block, int32_t mn_col, int32_t mn_extent,
                                      uint64_t* out);

/* kl_mma_instr_desc with the operand majors: 0 = K-major, 1 = MN-major. No counterpart in the
 * reference (K-major only). */
KL_API kl_status kl_mma_instr_desc_major(int32_t a_type, int32_t b_type, int32_t acc_type, int32_t m, int32_t n,
                                         int32_t a_major, int32_t b_major, uint32_t* out);

/* 128-byte TMA tensor map for a rank-`rank` row-major global tensor (shape/stride outermost
 * first, in elements) moved in tiles of tile_rows x tile_cols with the given swizzle. Needs a CUDA
 * driver (the encoding is the driver's). kernel_lib/include/kl/layout/tma_desc.hpp:100-164
 * (make_tma_desc / make_tma_load / make_tma_store). Same validation and messages. dtype KL_E3M2 /
 * KL_E2M3 (no counterpart in the reference): packed fp6 in global memory, a 16U6 map of 128-element
 * boxes (one byte per element in shared memory), with the driver's rules for that type checked. */
KL_API kl_status kl_make_tma_desc(int32_t dtype, int32_t tile_rows, int32_t tile_cols, int32_t swizzle_span, int32_t is_store,
                           const void* gmem, int32_t rank, const int64_t* shape, const int64_t* stride,
                           void* map_out);

#ifdef __cplusplus
}
#endif

#endif /* KL_GEMM_H_ */
