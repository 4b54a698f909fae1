// Host-side admission for the vq4 operations: the schema-1 plan of the
// reference (vq4_ops.rs:1-243, same order of checks, same refusal names and
// codes) and the schema-2 plan of this library's extension entry.
#pragma once

#include <array>
#include <cstdint>
#include <string>

namespace ack {

constexpr uint32_t kEntries = 16;
constexpr uint32_t kIndicesPerWord = 8;
constexpr uint32_t kWorkgroupSize = 64;          // vq4_ops.rs:18; names the reference grid
constexpr uint32_t kMaxValues = 1u << 28;        // vq4_ops.rs:19
constexpr uint32_t kMaxDim = 65536;              // vq4_ops.rs:20
constexpr uint64_t kMaxMatmulMacs = 1ull << 28;  // vq4_ops.rs:23
constexpr uint32_t kGridX = 65535;               // vq4_ops.rs:24
constexpr int kSlots = 8;                        // schema 2; schema 1 uses the first 6 slot positions

enum class Op : uint32_t {
  Encode = 0, Decode = 1, Matmul = 2, AdamW = 3,
  Dense = 16, Coded = 17, AdamwSample = 18, AdamwUsage = 19, AdamwEncode = 20,
  EncodeLarge = 21, DecodeLarge = 22, RepackTile32 = 23, AdamwFit = 24, Fit = 25,
  Residual = 26, ClipNorm = 27,
};

// Refusals. The schema-1 names are vq4_ops.rs:66-84; the schema-2 ones are
// this library's and are prefixed "vq2-".
enum class PlanError {
  None, Operation, Group, Entries, Flags, Reserved, Geometry, AddressLimit, WorkLimit,
  Capacity, NullIdentity, OutputAlias, StatusAlias, Dispatch,
  // schema 2 only
  Batch, Aux, Misaligned,
};

struct Plan {
  int schema = 1;                 // 1: 32-byte block, 6 slots; 2: 64-byte block, 8 slots
  std::array<uint32_t, 16> words{};
  Op op = Op::Encode;
  uint32_t group = 8;
  uint64_t m = 0, n = 0, k = 0;   // m carries the 64-bit value count of ops 21/22
  uint32_t flags = 0;
  uint32_t batch = 1;
  uint32_t aux0 = 0, aux1 = 0, aux2 = 0;
  // Required byte capacity per slot. Schema 1: [b0,b1,b2,b3,out,status];
  // schema 2: [in0,in1,in2,in3,in4,out0,out1,status].
  std::array<uint64_t, kSlots> required{};
  uint32_t work_items = 0;        // schema 1: the reference's dispatch accounting
  std::array<uint32_t, 3> dispatch{{0, 0, 0}};
  int nslots() const { return schema == 1 ? 6 : 8; }
  int first_output() const { return schema == 1 ? 4 : 5; }
  int status_slot() const { return schema == 1 ? 5 : 7; }
  // in4 is a workspace the operation writes: the device fits (ops 24, 25)
  // and the tensor-core dense product (op 16, flag 8)
  bool writes_in4() const {
    return schema == 2 && (op == Op::AdamwFit || op == Op::Fit || op == Op::Residual || op == Op::ClipNorm ||
                           (op == Op::Dense && (flags & 8u)));
  }
};

// Bytes of a packed code image of `values` values: ceil(ceil(values/g)/8) u32 words.
inline uint64_t packed_bytes(uint64_t values, uint32_t group) {
  return ((values + group - 1) / group + 7) / 8 * 4;
}
inline uint64_t packed_words(uint64_t values, uint32_t group) { return packed_bytes(values, group) / 4; }

// The tile32 layout of a coded N x K matrix (vectors along K, T = K/G a
// multiple of 32): rows grouped in tiles of 32 (the last tile padded with
// zero codes); within a tile, 16-byte chunk c (32 groups) of row r sits at
// ((tile * T/32 + c) * 32 + r % 32) * 16 bytes, so a warp reads chunk c of its
// 32 rows as one contiguous 512-byte line.
inline uint64_t tile32_bytes(uint64_t rows, uint64_t cols, uint32_t group) {
  return (rows + 31) / 32 * 32 * (cols / group) / 2;
}

// Workspace of the device codebook fit (op 24) per fitted book: the sample's
// nearest entries (one byte each, padded to 16), entry counts, whole-tensor
// usage counts and a flag word.
inline uint64_t fit_workspace_stride(uint32_t samples) { return (uint64_t(samples) + 15) / 16 * 16 + 160; }

// The tensor-core path of the dense product (op 16, flag 8) handles X rows in
// passes of at most kDenseTcMaxRows; a pass's projections P (bf16 hi and lo
// rows interleaved, 128 rows per 64-row tile of X, 16 K / G values each, per
// expert) live in the caller's workspace (slot in4).
constexpr uint32_t kDenseTcMaxRows = 128;
inline uint64_t dense_tc_workspace_bytes(uint64_t m, uint64_t k, uint32_t group, uint64_t batch) {
  const uint64_t mc = m < kDenseTcMaxRows ? m : kDenseTcMaxRows;
  return batch * ((mc + 63) / 64) * 128 * 16 * (k / group) * 2;
}

// The harness reductions (ops 26, 27) sum float64 partials of at most
// kReducePartials blocks, in a fixed order: their workspace (in4) holds the
// partials and, after them, the total.
constexpr uint32_t kReducePartials = 1024;
constexpr uint64_t kReduceWorkspace = (uint64_t(kReducePartials) + 1) * 8;

// Parse a plan block (32 bytes: schema 1, 64 bytes: schema 2). `slot` receives
// the offending slot for Capacity.
PlanError parse_plan(const uint8_t* bytes, size_t len, Plan* out);
// vq4_ops.rs:188-209: live identities (0 = null), capacities, alias rules.
PlanError validate_buffers(const Plan& p, const uint64_t* capacities, const uint64_t* ids, int* slot);
// vq4_ops.rs:211-222.
PlanError validate_dispatch(const Plan& p, const std::array<uint32_t, 3>& limits);

// "vq-..." / "vq2-..." refusal name; Capacity names its slot.
std::string plan_error_name(PlanError e, int schema, int slot);
// ACK_ERR_SIZE for Capacity/AddressLimit/WorkLimit, ACK_ERR_SHAPE otherwise (ffi.rs:6011-6018).
int32_t plan_error_code(PlanError e);

}  // namespace ack
