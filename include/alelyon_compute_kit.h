/*
 * alelyon_compute_kit.h -- the C ABI of the B200 vq4/v1 library
 * (libalelyon_compute_kit.so, built for sm_100a).
 *
 * This is the drop-in boundary for the reference's `vq4/v1` extension. The
 * first block of entries keeps the reference's C ABI (its Rust `ffi.rs`,
 * ABI version 14) symbol for symbol, with the same argument meaning, return
 * codes and refusal names, so that a binding written for the reference's
 * core + vq entries binds this library unchanged. Paths in the citations are
 * relative to the reference's `src/alelyon_compute_kit/_kit/`.
 *
 * Handles are ids, never addresses: a device handle is a process-wide
 * sequence number and a buffer handle is (device id << 32) | sequence. No
 * entry dereferences a handle; each is looked up in a registry and refused
 * by code when closed (ACK_ERR_CLOSED), foreign (ACK_ERR_FOREIGN) or freed
 * (ACK_ERR_FREED) -- the reference contract of ffi.rs:10-25.
 *
 * ACK_OK from an operator entry means the work was ENQUEUED on the device's
 * CUDA stream, not that it finished (ffi.rs:48-64). ack_download is the
 * synchronisation point; read the status word before trusting an output
 * (vq4.comp:5-8).
 */
#ifndef ALELYON_COMPUTE_KIT_H
#define ALELYON_COMPUTE_KIT_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Opaque handle types (ffi.rs: `AckDevice`, `Buffer`). Never dereferenced. */
typedef struct AckDevice AckDevice;
typedef struct AckBuffer AckBuffer;

/* Return codes, values of ffi.rs:726-760. */
#define ACK_OK 0
#define ACK_ERR_NULL (-1)
#define ACK_ERR_VULKAN (-2)          /* a driver error; here, a CUDA runtime error */
#define ACK_ERR_SHAPE (-3)
#define ACK_ERR_SIZE (-4)
#define ACK_ERR_LIVE_BUFFERS (-5)
#define ACK_ERR_CLOSED (-6)
#define ACK_ERR_FOREIGN (-7)
#define ACK_ERR_FREED (-8)
#define ACK_ERR_ABI (-9)
#define ACK_ERR_POISONED (-10)
#define ACK_ERR_UNSUPPORTED_OP (-11)
#define ACK_ERR_TIMING (-12)

#define ACK_ABI_VERSION 14u            /* ffi.rs:867 */
#define ACK_DEVICE_INFO_VERSION 1u     /* ack.py ACK_DEVICE_INFO_VERSION */
#define ACK_VQ_SCHEMA 1u               /* vq4_ops.rs:13 */
#define ACK_VQ_PUSH_BYTES 32u          /* vq4_ops.rs:15 */
#define ACK_VQ2_SCHEMA 1u              /* schema of the B200 extension entry ack_vq2 */
#define ACK_VQ2_PLAN_BYTES 64u
#define ACK_VQ2_SLOTS 8u

/* Status word bits written by every vq kernel (vq4.comp:5-8). */
#define ACK_VQ_STATUS_NONFINITE 1u
#define ACK_VQ_STATUS_LAYOUT 2u
#define ACK_VQ_STATUS_OPTIMIZER 4u
/* B200 extension, no reference counterpart: a pipelined kernel's bounded
 * wait on one of its own barriers ran out; the outputs are not valid. */
#define ACK_VQ_STATUS_STALLED 8u

/* What ack_abi_info reports (ffi.rs:1009-1057, 96 bytes, same layout). This
 * library carries none of the reference's twelve dense operator families, so
 * `operators` and every op_schema_* field are 0; the vq extension announces
 * itself through ack_vq_schema / ack_vq2_schema, as in the reference. */
typedef struct AckAbiInfo {
    uint32_t size;
    uint32_t version;
    uint64_t operators;
    uint64_t shaders;   /* FNV-1a over the embedded CUDA kernel manifest */
    uint64_t build;     /* FNV-1a over the library version and `shaders` */
    uint32_t op_schema_matmul_bf16;
    uint32_t op_schema_cast;
    uint32_t capability_streams;
    uint32_t capability_rng;
    uint32_t capability_optimizer;
    uint32_t capability_serialization;
    uint32_t op_schema_matmul_f32;
    uint32_t op_schema_pointwise;
    uint32_t op_schema_reduce;
    uint32_t op_schema_rowwise;
    uint32_t op_schema_loss;
    uint32_t op_schema_embedding;
    uint32_t op_schema_matmul_f16;
    uint32_t op_schema_index;
    uint32_t op_schema_convert;
    uint32_t op_schema_intwise;
} AckAbiInfo;

/* What ack_device_info reports (ffi.rs:1223-1255, 616 bytes, same layout),
 * filled from the CUDA device: vendor 0x10DE, the device UUID, warp size as
 * `subgroup_size`, CUDA grid/block limits as the workgroup limits. */
typedef struct AckDeviceInfo {
    uint32_t size;
    uint32_t version;
    uint32_t api_version;
    uint32_t driver_version_raw;
    uint32_t driver_id;
    uint32_t vendor_id;
    uint32_t device_id;
    uint32_t device_type;
    uint8_t device_uuid[16];
    uint8_t driver_uuid[16];
    uint64_t features;
    uint32_t subgroup_size;
    uint32_t timestamp_valid_bits;
    float timestamp_period_ns;
    uint32_t max_push_constant_bytes;
    uint64_t device_local_bytes;
    uint64_t max_storage_buffer_bytes;
    uint32_t max_workgroup_invocations;
    uint32_t max_workgroup_count[3];
    uint32_t max_workgroup_size[3];
    uint32_t matmul_tile;
    uint32_t matmul_k_multiple;
    uint32_t matmul_layouts;
    uint32_t matmul_operand_dtype;
    uint32_t matmul_result_dtype;
    uint32_t cast_modes;
    uint32_t reserved;
    uint64_t identity;
    char device_name[256];
    char driver_name[64];
    char driver_info[128];
} AckDeviceInfo;

/* ---- core device ABI (the subset the reference binding loads, ack.py:714-739) ---- */

/* ffi.rs:1981 ack_abi_info. ACK_ERR_ABI when `size` < sizeof(AckAbiInfo). */
int32_t ack_abi_info(AckAbiInfo *out, size_t size);
/* ffi.rs:2410 ack_device_info. */
int32_t ack_device_info(const AckDevice *dev, AckDeviceInfo *out, size_t size);
/* ffi.rs:2037 ack_open: opens the CUDA device ACK_DEVICE names ("gpu", "gpu:<n>",
 * "any", "any:<n>"; device_choice.rs:11-22), else the thread's current CUDA
 * device. Null with ack_last_error set on failure ("cpu" is refused: this
 * build has no CPU device). */
AckDevice *ack_open(void);
/* ffi.rs:2365 ack_close: ACK_ERR_LIVE_BUFFERS while buffers are live. */
int32_t ack_close(AckDevice *dev);
/* ffi.rs:3296 ack_device_name. */
int32_t ack_device_name(const AckDevice *dev, char *out, size_t len);
/* ffi.rs:2741 ack_live_objects: CUDA objects this device holds (its stream,
 * live buffers). */
int32_t ack_live_objects(const AckDevice *dev, int64_t *out);
/* ffi.rs:3276 ack_leaked_on_poison: buffers left allocated because the
 * device was poisoned when they were freed. */
int32_t ack_leaked_on_poison(const AckDevice *dev, uint64_t *out);
/* ffi.rs:3325 ack_last_error: this thread's last message. */
int32_t ack_last_error(char *out, size_t len);
/* ffi.rs:3345 ack_buffer_alloc: a device buffer (cudaMalloc); null on failure. */
AckBuffer *ack_buffer_alloc(const AckDevice *dev, uint64_t bytes);
/* ffi.rs:3413 ack_buffer_free. */
int32_t ack_buffer_free(const AckDevice *dev, AckBuffer *buf);
/* ffi.rs:3477 ack_upload: `len` must equal the buffer size. */
int32_t ack_upload(const AckDevice *dev, const AckBuffer *buf, const void *data, size_t len);
/* ffi.rs:3525 ack_download: waits for all enqueued work, then copies. */
int32_t ack_download(const AckDevice *dev, const AckBuffer *buf, void *data, size_t len);

/* ---- vq4/v1 extension (ffi.rs:6004-6151, vq4_ops.rs) ---- */

/* ffi.rs:6006 ack_vq_schema: always 1. */
uint32_t ack_vq_schema(void);
/* ffi.rs:6037 ack_vq: encode (op 0), decode (1), packed-pair matmul (2),
 * decoded-state AdamW (3). `plan` is 8 little-endian u32
 * [op, m, n, k, group, 16, flags, 0]; admission, slot sizes, refusal names
 * and codes are those of vq4_ops.rs:111-222, including the 2^28 value and
 * matmul-MAC bounds. Results follow vq4.comp: encode picks the float64
 * nearest code vector with lowest-index ties (the reference CPU encoder,
 * vq.py:154-179), decode is exact, op 2 sums fl32(a*b) in k order with
 * separately rounded adds, op 3 is AdamW in FP32 in the shader's order. */
int32_t ack_vq(const AckDevice *dev, const AckBuffer *b0, const AckBuffer *b1, const AckBuffer *b2,
               const AckBuffer *b3, const AckBuffer *out, const AckBuffer *status,
               const uint8_t *plan, size_t plan_len);

/* ---- B200 extension of vq4 (schema 2). No counterpart in the reference's
 * C ABI; these are the north-star operations the reference lacks
 * (dense-activation product, unbounded coded product, fused coded-state
 * AdamW, 64-bit encode/decode). ---- */

/* Plan operations of ack_vq2 / ack_vq_launch with a 64-byte plan. */
#define ACK_VQ2_DENSE 16u        /* Y_b = X_b * op(decode W_b), batch b of independent products */
#define ACK_VQ2_CODED 17u        /* C = op(decode A) * op(decode B), no MAC bound */
#define ACK_VQ2_ADAMW_SAMPLE 18u /* AdamW values of the calibration sample vectors */
#define ACK_VQ2_ADAMW_USAGE 19u  /* entries a trial book selects over one updated state */
#define ACK_VQ2_ADAMW_ENCODE 20u /* decode -> AdamW -> encode W', M', V' in one pass */
#define ACK_VQ2_ENCODE 21u       /* encode with a 64-bit value count */
#define ACK_VQ2_DECODE 22u       /* decode with a 64-bit value count */
#define ACK_VQ2_REPACK_TILE32 23u /* canonical N x K images -> the tile32 layout op 16 reads */
#define ACK_VQ2_ADAMW_FIT 24u    /* fit_codebook of W', M', V' on the device (warm start), bit for bit the CPU fit */
#define ACK_VQ2_FIT 25u          /* fit_codebook of one tensor on the device, bit for bit the CPU function */
#define ACK_VQ2_RESIDUAL 26u     /* harness residual: r = P - decode(T), r * s and the float64 sum of r^2 */
#define ACK_VQ2_CLIP 27u         /* harness clip: float64 norm, g * fl32(min(1, max / (norm + 1e-6))) */

/* Flags of ACK_VQ2_DENSE: bit 1 = W stored N x K (vectors along K); bit 2 =
 * W given in the tile32 layout (requires bit 1 and (K / group) % 32 == 0):
 * rows in tiles of 32, the last padded with zero codes; 16-byte chunk c of
 * row r at byte ((r / 32) * (K / group / 32) + c) * 512 + (r % 32) * 16. */
#define ACK_VQ2_DENSE_NT 2u
#define ACK_VQ2_DENSE_TILE32 4u
/* bit 3: the tensor-core kernel (one-hot codes times the bf16 hi + lo
 * projections of X on the entries); requires bit 1, the canonical layout
 * and (K / group) % 32 == 0; in4 is its workspace, written:
 * batch x ceil(min(M, 128) / 64) x 128 x 16 K / group x 2 bytes. */
#define ACK_VQ2_DENSE_TENSOR 8u

uint32_t ack_vq2_schema(void);

/* The kernel manifest, the CUDA counterpart of the reference's vq4 entry in
 * K/kernels/MANIFEST.json:2137-2144: a NUL-terminated JSON object with the
 * sha256 of every library source, the kernels each defines, the nvcc
 * release and flags and the arch (sm_100a). `*needed` receives the size
 * including the NUL; `out` may be null to ask for it. ACK_ERR_SIZE if `len`
 * is short. AckAbiInfo.shaders is the FNV-1a hash of the same text. */
int32_t ack_kernel_manifest(char *out, size_t len, size_t *needed);
/* `plan` is 16 little-endian u32 [op, m, n, k, group, 16, flags, 0, batch,
 * aux0, aux1, aux2, 0, 0, 0, 0]; `slots` is ACK_VQ2_SLOTS buffer handles
 * [in0, in1, in2, in3, in4, out0, out1, status]; a slot the operation does
 * not use may be null; refusals are named "vq2-..." and carry the schema-1
 * codes. Slots per operation (in0, in1, in2, in3 -> out0, out1):
 *   16 dense      X (batch x M x K f32), W codes (batch x words), W books
 *                 (batch x 16 x g) -> Y (batch x M x N)
 *   17 coded      A codes, A book, B codes, B book -> C (M x N)
 *   18 sample     W/M/V/G images per expert, their 4 books, 7 coefficients,
 *                 aux0 = S sample vector positions -> (batch x 3 x S x g) f32
 *   19 usage      as 18, trial book; aux0 = state, aux1 = expert -> 16 u32
 *   20 encode     as 18, new books (batch x 3 x 16 x g) -> codes
 *                 (batch x 3 x words), changed (batch u32)
 *   21/22         values or codes, book -> codes or values
 *   23 repack     canonical codes (batch x words) -> tile32 codes
 *   24 fit        as 18, op 18's samples (batch x 3 x S x g), in4 = workspace
 *                 (batch x 3 x (ceil16(S) + 160) bytes, written); flags = 1
 *                 (warm start), aux0 = S, aux1 = iterations -> fitted books
 *                 (batch x 3 x 16 x g)
 *   25 fit        values (count = m + aux2 << 32), warm book (flags bit 0),
 *                 u32 sample positions then 16 cold-start sample rows,
 *                 in4 = workspace (S x g x 4 + ceil16(S) + 160 bytes,
 *                 written); aux0 = S, aux1 = iterations -> book (16 x g)
 *   26 residual   prediction (m f32), target codes, target book, in4 =
 *                 workspace ((1024 + 1) x 8 bytes, written, 8-byte aligned);
 *                 aux0 = the FP32 bits of s -> r * s (m f32), sum r^2 (f64)
 *   27 clip       gradient (m f32), in4 = workspace as 26; aux0/aux1 = the
 *                 low/high words of the float64 max norm -> g * fl32(scale)
 *                 (m f32), [norm, scale] (2 f64) */
int32_t ack_vq2(const AckDevice *dev, const AckBuffer *const *slots, size_t nslots,
                const uint8_t *plan, size_t plan_len);

/* The grouped dense product (op 16) from and to host memory, pipelined: no
 * counterpart in the reference (its products take and return device
 * buffers one call at a time). `plan` is an op-16 plan for the whole batch;
 * `codes` and `books` are device buffers holding the weights (canonical or
 * tile32, as the flags say), `x` (batch x M x K f32) and `y` (batch x M x N
 * f32) host memory. The experts run in `parts` contiguous ranges (0: the
 * library chooses): the parts' X are copied in back to back on one stream,
 * part c computes once its X is in and its Y is copied out on a third stream
 * once computed, so the copies and the products overlap (host memory must be
 * page-locked for the copies to be asynchronous). Returns when all of `y` is written; `*status_out` (not
 * null) receives the status word of the whole product, read once; bit 1
 * there covers a nonfinite X or product (X is not scanned on the host). The
 * device scratch (all of X and Y, and two tensor-core workspaces when flag 8
 * is set) is allocated on first use, grows to the largest call's need and is
 * kept by the device until ack_close. */
int32_t ack_vq2_dense_host(const AckDevice *dev, const uint8_t *plan, size_t plan_len, const AckBuffer *codes,
                           const AckBuffer *books, const float *x, float *y, uint32_t parts, uint32_t *status_out);

/* Device-pointer form of both entries, for callers whose data already lives
 * in device memory (a PyTorch tensor, an NCCL buffer): the same plan, the
 * same admission and refusals, operands given as CUDA device pointers with
 * their byte capacities, work enqueued on the caller's CUDA stream `stream`
 * (a cudaStream_t; null = the legacy default stream) on the current device.
 * A 32-byte plan uses slots [b0, b1, b2, b3, out, status]; a 64-byte plan the
 * ack_vq2 slots. Every non-null pointer must be 4-byte aligned; the
 * 128-bit kernels (tile32 codes) also want 16-byte alignment. */
typedef struct AckVqOperands {
    uint32_t size;      /* sizeof(AckVqOperands) */
    uint32_t nslots;    /* 6 for a schema-1 plan, 8 for a schema-2 plan */
    uint64_t bytes[8];
    void *ptr[8];
} AckVqOperands;
int32_t ack_vq_launch(const uint8_t *plan, size_t plan_len, const AckVqOperands *ops, void *stream);

/* Encode without any allocation. No counterpart in the reference: an entry
 * for callers that cannot allocate device memory, because their host owns
 * every device allocation (an engine or server with its own allocator) or
 * because an allocation at that point would stall or be refused. It encodes
 * `batch` tensors of `count` values each (x: batch x count floats, books:
 * batch x 16 x group, codes: batch x ceil(ceil(count/group)/8) u32 words,
 * status: one u32 the caller has cleared), all device pointers, 4-byte
 * aligned, on `stream` (a cudaStream_t) of the current device; the codes are
 * the bytes ack_vq_launch's encode (op 21) produces. The only device memory
 * it uses besides these is a fixed 139,264-byte array in the library, held
 * by every GPU that loads it until exit, which limits a call to batch <= 64
 * (ACK_ERR_SIZE beyond). The first call on a device looks that array's
 * address up (cudaGetSymbolAddress); make that first call before any stream
 * capture. Every call shares the array: calls that may overlap on the GPU
 * (other streams, other threads) race and must be serialised by the caller.
 * ACK_ERR_NULL / ACK_ERR_SHAPE for null, misaligned or overlapping operands
 * and a group other than 8, 16, 32. */
int32_t ack_vq_encode_noalloc(const float *x, uint64_t count, uint32_t batch, const float *books, uint32_t group,
                              uint32_t *codes, uint32_t *status, void *stream);

/* ---- host-only planner introspection (the public methods of the
 * reference's VqPlan, vq4_ops.rs:111-243, which its Rust tests call
 * directly). No device is touched. Each returns ACK_OK or the code ack_vq
 * would return, with the refusal name in ack_last_error. ---- */
int32_t ack_vq_plan_probe(const uint8_t *plan, size_t plan_len, uint64_t required_bytes[8],
                          uint32_t *work_items, uint32_t dispatch[3]);
int32_t ack_vq_plan_validate_buffers(const uint8_t *plan, size_t plan_len,
                                     const uint64_t *capacities, const uint64_t *ids, size_t n);
int32_t ack_vq_plan_validate_dispatch(const uint8_t *plan, size_t plan_len, const uint32_t limits[3]);

/* ---- the NF4 comparator (the adjacent 4-bit format of the same kit, for
 * comparison with vq4) ----
 * nf4-decode/v1 and nf4-gemv/v1 with the reference's names, arguments,
 * refusal names and codes (ffi.rs:7365 ack_nf4_decode, :8017 ack_gemv_nf4;
 * planners nf4_ops.rs:158-204, :515-569; the law in kernels/nf4_decode.comp
 * and nf4_gemv.comp). Buffers: packed (two indices a byte, high nibble
 * first), absmax_q (a byte a block of 64 values), absmax2 (f32 a nested
 * block of 256 blocks), tables (the 16 code values then the 256 map values,
 * f32), starts (int64 a member), offsets (f32 a member), ids (int64 a
 * selected member; unread and may be null when `selected` is 0), out.
 * storage: 0 f32, 1 bf16, 2 fp16; elem: 0 bf16, 1 fp16. The work is enqueued
 * on the device's stream; `ms_out`, when given, reads NaN. */
int32_t ack_nf4_decode(const AckDevice *dev, const AckBuffer *packed, const AckBuffer *absmax_q,
                       const AckBuffer *absmax2, const AckBuffer *tables, const AckBuffer *starts,
                       const AckBuffer *offsets, const AckBuffer *ids, const AckBuffer *out, uint32_t n,
                       uint32_t members, uint32_t selected, uint32_t member_values, uint32_t src_base,
                       uint32_t storage, double *ms_out);
/* C[first + m, :] = A[first + m, :] . W^T for each group (first row, rows,
 * weight base: three u32 words) of `groups_table`; A is `rows` x `lda`
 * 16-bit words (lda 0: K), C `rows` x `n` f32. */
int32_t ack_gemv_nf4(const AckDevice *dev, const AckBuffer *a, const AckBuffer *packed, const AckBuffer *absmax_q,
                     const AckBuffer *absmax2, const AckBuffer *tables, const AckBuffer *starts,
                     const AckBuffer *offsets, const AckBuffer *groups_table, const AckBuffer *c, uint32_t rows,
                     uint32_t max_rows, uint32_t n, uint32_t k, uint32_t lda, uint32_t groups, uint32_t members,
                     uint32_t src_base, uint32_t elem, double *ms_out);
/* Device-pointer forms (no counterpart in the reference): the operands of
 * the entries above in the same order as CUDA device pointers with their
 * byte sizes, enqueued on the cudaStream_t `stream` of the current device. */
int32_t ack_nf4_decode_launch(void *const *ptrs, const uint64_t *bytes, uint32_t n, uint32_t members,
                              uint32_t selected, uint32_t member_values, uint32_t src_base, uint32_t storage,
                              void *stream);
int32_t ack_gemv_nf4_launch(void *const *ptrs, const uint64_t *bytes, uint32_t rows, uint32_t max_rows, uint32_t n,
                            uint32_t k, uint32_t lda, uint32_t groups, uint32_t members, uint32_t src_base,
                            uint32_t elem, void *stream);

/* ---- peer stores between ranks (no counterpart in the reference: its kit
 * has no multi-GPU layer). One process per GPU; each rank allocates a buffer
 * others map through CUDA IPC (no multicast object), exchanges the 64-byte
 * handles (e.g. over torch.distributed) and opens the others'. ---- */
int32_t ack_peer_alloc(uint64_t bytes, void **ptr, uint8_t *handle64);   /* zeroed, current device */
int32_t ack_peer_open(const uint8_t *handle64, void **ptr);
int32_t ack_peer_close(void *ptr);
int32_t ack_peer_free(void *ptr);
/* ack_vq_launch's op-16 plan (M = 1, W stored N x K, canonical codes, the
 * byte-pair kernel's shapes; ACK_ERR_UNSUPPORTED_OP otherwise) whose outputs
 * are also stored into `npeers` (at most 7) other ranks' slots at Y's offsets;
 * its blocks fence at system scope before they exit. */
int32_t ack_vq_dense_peers(const uint8_t *plan, size_t plan_len, const AckVqOperands *ops, float *const *peers,
                           uint32_t npeers, void *stream);
/* After the stream's earlier work, store `epoch` (release, system scope) into
 * slot `rank` of each of the `world` flag arrays (u32 per sender). */
int32_t ack_peer_signal(uint32_t *const *flags, uint32_t world, uint32_t rank, uint32_t epoch, void *stream);
/* Wait until each of this rank's `world` flags has reached `epoch` (epochs
 * only grow), at most `polls` polls a flag (0: 2^24, about two seconds);
 * a wait that runs out ORs ACK_VQ_STATUS_STALLED into `status`. */
int32_t ack_peer_wait(const uint32_t *flags, uint32_t world, uint32_t epoch, uint32_t *status, uint32_t polls,
                      void *stream);

/* ---- test-only host fault injection (the reference's `ack_inject_fault`,
 * ffi.rs:3449, behind its `fault-injection` feature). Refused unless the
 * process environment has ACK_FAULT_INJECTION=1. kind 0: the next stream
 * synchronisation reports `code` (a cudaError_t) after the real wait ran;
 * kind 1: the next buffer allocation reports cudaErrorMemoryAllocation after
 * freeing what it allocated; kind 2: the next tensor-core encode launch (in
 * this process) runs a stall test, code 1 its TMA producer issuing no load,
 * code 2 its consumers taking no accumulator: the bounded waits that nothing
 * will satisfy run out after a short bound, the kernel sets
 * ACK_VQ_STATUS_STALLED, waits for its own loads and MMAs in flight and
 * returns, and the context stays usable. No fault, trap or hang is caused on
 * the GPU. ---- */
int32_t ack_inject_fault(const AckDevice *dev, int32_t kind, int32_t code);

#ifdef __cplusplus
}
#endif

#endif /* ALELYON_COMPUTE_KIT_H */
