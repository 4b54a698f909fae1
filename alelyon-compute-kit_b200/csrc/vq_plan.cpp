// Admission for the vq4 operations. The schema-1 rules restate the
// reference planner vq4_ops.rs:111-222 check for check; the schema-2 rules
// cover this library's extension operations.
#include "vq_plan.hpp"

#include <cstring>

#include "alelyon_compute_kit.h"

namespace ack {
namespace {

uint32_t le32(const uint8_t* p) {
  return uint32_t(p[0]) | (uint32_t(p[1]) << 8) | (uint32_t(p[2]) << 16) | (uint32_t(p[3]) << 24);
}

bool valid_group(uint32_t g) { return g == 8 || g == 16 || g == 32; }

uint64_t div_up(uint64_t x, uint64_t d) { return (x + d - 1) / d; }

// vq4_ops.rs:101-108: a u32 product bounded by MAX_VALUES.
PlanError product(uint32_t a, uint32_t b, uint32_t* out) {
  uint64_t v = uint64_t(a) * uint64_t(b);
  if (v > kMaxValues) return PlanError::AddressLimit;
  *out = uint32_t(v);
  return PlanError::None;
}

void set_dispatch(Plan* p) {
  // vq4_ops.rs:173-175: the reference's 64-wide workgroup grid, kept so the
  // dispatch refusal and the planner probes answer as the reference does.
  uint32_t groups = uint32_t(div_up(p->work_items, kWorkgroupSize));
  uint32_t x = groups < kGridX ? groups : kGridX;
  p->dispatch = {x, x ? uint32_t(div_up(groups, x)) : 0u, 1u};
}

PlanError parse_schema1(Plan* p) {
  const auto& w = p->words;
  uint32_t op = w[0], m = w[1], n = w[2], k = w[3], group = w[4], entries = w[5], flags = w[6],
           reserved = w[7];
  if (op > 3) return PlanError::Operation;
  if (!valid_group(group)) return PlanError::Group;
  if (entries != kEntries) return PlanError::Entries;
  if (reserved != 0) return PlanError::Reserved;
  if ((op == 2 && flags > 3) || (op != 2 && flags != 0)) return PlanError::Flags;
  if (m == 0 || n == 0 || k == 0) return PlanError::Geometry;
  p->op = Op(op);
  p->group = group;
  p->m = m;
  p->n = n;
  p->k = k;
  p->flags = flags;
  const uint64_t book = uint64_t(kEntries * group) * 4;
  if (op != 2) {
    if (n != 1 || k != 1) return PlanError::Geometry;
    if (m > kMaxValues) return PlanError::AddressLimit;
    uint64_t packed = packed_bytes(m, group);
    uint64_t dense = uint64_t(m) * 4;
    if (op == 0) {
      p->required = {dense, book, 0, 0, packed, 4, 0, 0};
      p->work_items = uint32_t(packed / 4);
    } else if (op == 1) {
      p->required = {packed, book, 0, 0, dense, 4, 0, 0};
      p->work_items = m;
    } else {
      uint32_t unused;
      PlanError e = product(m, 3, &unused);
      if (e != PlanError::None) return e;
      p->required = {4 * packed, 4 * book, 7 * 4, 0, 3 * dense, 4, 0, 0};
      p->work_items = m;
    }
  } else {
    if (m > kMaxDim || n > kMaxDim || k > kMaxDim) return PlanError::Geometry;
    uint32_t a, b, c;
    PlanError e = product(m, k, &a);
    if (e == PlanError::None) e = product(k, n, &b);
    if (e == PlanError::None) e = product(m, n, &c);
    if (e != PlanError::None) return e;
    if (uint64_t(c) * uint64_t(k) > kMaxMatmulMacs) return PlanError::WorkLimit;
    p->required = {packed_bytes(a, group), book, packed_bytes(b, group), book, uint64_t(c) * 4, 4, 0, 0};
    p->work_items = c;
  }
  set_dispatch(p);
  return PlanError::None;
}

constexpr uint64_t kMaxDim2 = 1ull << 20;       // per-axis bound of the schema-2 products
constexpr uint64_t kMaxOperand2 = 1ull << 34;   // values per operand of one schema-2 product
constexpr uint64_t kMaxLarge = 1ull << 36;      // values of one ops-21/22 call
constexpr uint32_t kMaxSamples = 65536;         // fit_codebook's sample bound (vq.py:202)

PlanError parse_schema2(Plan* p) {
  const auto& w = p->words;
  uint32_t op = w[0], group = w[4], entries = w[5], flags = w[6], reserved = w[7];
  if (op < 16 || op > 27) return PlanError::Operation;
  if (!valid_group(group)) return PlanError::Group;
  if (entries != kEntries) return PlanError::Entries;
  if (reserved != 0 || w[12] || w[13] || w[14] || w[15]) return PlanError::Reserved;
  p->op = Op(op);
  p->group = group;
  p->m = w[1];
  p->n = w[2];
  p->k = w[3];
  p->flags = flags;
  p->batch = w[8];
  p->aux0 = w[9];
  p->aux1 = w[10];
  p->aux2 = w[11];
  const uint64_t book = uint64_t(kEntries) * group * 4;
  const uint64_t E = p->batch;
  switch (p->op) {
    case Op::Dense: {
      // flag bit 1: W stored N x K (groups along K); clear: W stored K x N.
      // flag bit 2: W is in the tile32 layout (needs bit 1, K % G == 0 and
      // (K / G) % 32 == 0).
      // flag bit 3: the tensor-core kernel, with its workspace in in4 (needs
      // bit 1, the canonical layout, K % G == 0 and (K / G) % 32 == 0).
      if (flags & ~14u) return PlanError::Flags;
      if ((flags & 4u) && (!(flags & 2u) || p->k % group || (p->k / group) % 32)) return PlanError::Flags;
      if ((flags & 8u) && (!(flags & 2u) || (flags & 4u) || p->k % group || (p->k / group) % 32))
        return PlanError::Flags;
      if (p->aux0 || p->aux1 || p->aux2) return PlanError::Aux;
      if (!p->m || !p->n || !p->k) return PlanError::Geometry;
      if (!E) return PlanError::Batch;
      if (p->m > kMaxDim2 || p->n > kMaxDim2 || p->k > kMaxDim2) return PlanError::Geometry;
      if (p->m * p->k > kMaxOperand2 || p->n * p->k > kMaxOperand2 || p->m * p->n > kMaxOperand2)
        return PlanError::AddressLimit;
      uint64_t wb = (flags & 4u) ? tile32_bytes(p->n, p->k, group) : packed_bytes(p->n * p->k, group);
      const uint64_t ws = (flags & 8u) ? dense_tc_workspace_bytes(p->m, p->k, group, E) : 0;
      p->required = {E * p->m * p->k * 4, E * wb, E * book, 0, ws, E * p->m * p->n * 4, 0, 4};
      break;
    }
    case Op::RepackTile32: {
      // canonical N x K image (m = N, k = K) -> tile32 layout, batch of E
      if (flags) return PlanError::Flags;
      if (p->aux0 || p->aux1 || p->aux2) return PlanError::Aux;
      if (!p->m || p->n != 1 || !p->k) return PlanError::Geometry;
      if (p->k % group || (p->k / group) % 32) return PlanError::Geometry;
      if (!E) return PlanError::Batch;
      if (p->m > kMaxDim2 || p->k > kMaxDim2) return PlanError::Geometry;
      p->required = {E * packed_bytes(p->m * p->k, group), 0, 0, 0, 0, E * tile32_bytes(p->m, p->k, group), 0, 4};
      break;
    }
    case Op::Coded: {
      if (flags > 3) return PlanError::Flags;
      if (p->aux0 || p->aux1 || p->aux2) return PlanError::Aux;
      if (!p->m || !p->n || !p->k) return PlanError::Geometry;
      if (E != 1) return PlanError::Batch;
      if (p->m > kMaxDim2 || p->n > kMaxDim2 || p->k > kMaxDim2) return PlanError::Geometry;
      if (p->m * p->k > kMaxOperand2 || p->n * p->k > kMaxOperand2 || p->m * p->n > kMaxOperand2)
        return PlanError::AddressLimit;
      p->required = {packed_bytes(p->m * p->k, group), book, packed_bytes(p->k * p->n, group), book,
                     0, p->m * p->n * 4, 0, 4};
      break;
    }
    case Op::AdamwSample:
    case Op::AdamwUsage:
    case Op::AdamwEncode: {
      if (flags) return PlanError::Flags;
      if (!p->m || p->n != 1 || p->k != 1) return PlanError::Geometry;
      if (p->m > kMaxValues) return PlanError::AddressLimit;
      if (!E) return PlanError::Batch;
      const uint64_t words = packed_bytes(p->m, group);
      const uint64_t states = E * 4 * words, books = E * 4 * book, coefs = E * 7 * 4;
      if (p->op == Op::AdamwSample) {
        if (p->aux1 || p->aux2) return PlanError::Aux;
        if (!p->aux0 || p->aux0 > kMaxSamples || p->aux0 > p->m / group) return PlanError::Aux;
        p->required = {states, books, coefs, uint64_t(p->aux0) * 4, 0,
                       E * 3 * uint64_t(p->aux0) * group * 4, 0, 4};
      } else if (p->op == Op::AdamwUsage) {
        if (p->aux0 > 2 || p->aux1 >= E || p->aux2) return PlanError::Aux;
        if (p->m < group) return PlanError::Geometry;  // needs one complete vector
        p->required = {states, books, coefs, book, 0, kEntries * 4, 0, 4};
      } else {
        if (p->aux0 || p->aux1 || p->aux2) return PlanError::Aux;
        p->required = {states, books, coefs, E * 3 * book, 0, E * 3 * words, E * 4, 4};
      }
      break;
    }
    case Op::AdamwFit: {
      // fit_codebook (vq.py:182-257) of W', M', V' on the device, warm-started
      // from the current books (flag bit 0, the VQAdamW case): aux0 sample
      // vectors (op 18's output), aux1 Lloyd iterations.
      if (flags != 1u) return PlanError::Flags;
      if (!p->m || p->n != 1 || p->k != 1) return PlanError::Geometry;
      if (p->m > kMaxValues) return PlanError::AddressLimit;
      if (!E) return PlanError::Batch;
      if (!p->aux0 || p->aux0 > kMaxSamples || p->aux0 > p->m / group || p->aux1 > 32 || p->aux2)
        return PlanError::Aux;
      const uint64_t words = packed_bytes(p->m, group);
      p->required = {E * 4 * words, E * 4 * book, E * 7 * 4, E * 3 * uint64_t(p->aux0) * group * 4,
                     E * 3 * fit_workspace_stride(p->aux0), E * 3 * book, 0, 4};
      break;
    }
    case Op::Fit: {
      // fit_codebook (vq.py:182-257) of one tensor of count = m + aux2 << 32
      // values: aux0 sample vectors at the positions in in2 (followed by the
      // 16 cold-start rows of the sample), aux1 Lloyd iterations; flag bit 0:
      // warm start from the book in in1. in4: workspace (the sample, then the
      // fit's bookkeeping).
      if (flags & ~1u) return PlanError::Flags;
      if (p->n != 1 || p->k != 1) return PlanError::Geometry;
      if (E != 1) return PlanError::Batch;
      const uint64_t count = uint64_t(w[1]) | (uint64_t(p->aux2) << 32);
      if (count < group) return PlanError::Geometry;
      if (count > kMaxLarge) return PlanError::AddressLimit;
      p->m = count;
      if (!p->aux0 || p->aux0 > kMaxSamples || p->aux0 > count / group || p->aux1 > 32) return PlanError::Aux;
      const uint64_t sample_bytes = uint64_t(p->aux0) * group * 4;
      p->required = {count * 4, (flags & 1u) ? book : 0, (uint64_t(p->aux0) + 16) * 4, 0,
                     sample_bytes + fit_workspace_stride(p->aux0), book, 0, 4};
      break;
    }
    case Op::EncodeLarge:
    case Op::DecodeLarge: {
      if (flags) return PlanError::Flags;
      if (p->n != 1 || p->k != 1) return PlanError::Geometry;
      if (E != 1 || p->aux1 || p->aux2) return E != 1 ? PlanError::Batch : PlanError::Aux;
      uint64_t count = uint64_t(w[1]) | (uint64_t(p->aux0) << 32);
      if (!count) return PlanError::Geometry;
      if (count > kMaxLarge) return PlanError::AddressLimit;
      p->m = count;
      uint64_t packed = packed_bytes(count, group), dense = count * 4;
      if (p->op == Op::EncodeLarge)
        p->required = {dense, book, 0, 0, 0, packed, 0, 4};
      else
        p->required = {packed, book, 0, 0, 0, dense, 0, 4};
      break;
    }
    case Op::Residual: {
      // The harness residual (harness.py:186-193): r = prediction -
      // decode(target) over count = m values (in0 f32, in1/in2 the target's
      // codes and book); out0 = r * s with s the FP32 bit pattern in aux0
      // (2 / count), out1 = the float64 sum of r^2 (one value); in4 holds the
      // reduction's partials.
      if (flags) return PlanError::Flags;
      if (!p->m || p->n != 1 || p->k != 1) return PlanError::Geometry;
      if (E != 1) return PlanError::Batch;
      if (p->aux1 || p->aux2) return PlanError::Aux;
      if (p->m > kMaxOperand2) return PlanError::AddressLimit;
      p->required = {p->m * 4, packed_bytes(p->m, group), book, 0, kReduceWorkspace, p->m * 4, 8, 4};
      break;
    }
    case Op::ClipNorm: {
      // The harness clip (harness.py:194-200): norm = sqrt(sum g^2) in
      // float64 over count = m values of in0, scale = min(1, max_norm /
      // (norm + 1e-6)) with max_norm the float64 whose bits are aux0 (low)
      // and aux1 (high); out0 = g * fl32(scale), out1 = [norm, scale]
      // (float64); in4 holds the reduction's partials.
      if (flags) return PlanError::Flags;
      if (!p->m || p->n != 1 || p->k != 1) return PlanError::Geometry;
      if (E != 1) return PlanError::Batch;
      if (p->aux2) return PlanError::Aux;
      if (p->m > kMaxOperand2) return PlanError::AddressLimit;
      p->required = {p->m * 4, 0, 0, 0, kReduceWorkspace, p->m * 4, 16, 4};
      break;
    }
    default:
      return PlanError::Operation;
  }
  p->work_items = 0;
  p->dispatch = {1, 1, 1};
  return PlanError::None;
}

}  // namespace

PlanError parse_plan(const uint8_t* bytes, size_t len, Plan* out) {
  Plan p;
  if (len == ACK_VQ_PUSH_BYTES) {
    p.schema = 1;
    for (int i = 0; i < 8; ++i) p.words[i] = le32(bytes + 4 * i);
    PlanError e = parse_schema1(&p);
    *out = p;
    return e;
  }
  p.schema = 2;
  for (int i = 0; i < 16; ++i) p.words[i] = le32(bytes + 4 * i);
  PlanError e = parse_schema2(&p);
  *out = p;
  return e;
}

PlanError validate_buffers(const Plan& p, const uint64_t* capacities, const uint64_t* ids, int* slot) {
  const int n = p.nslots();
  if (p.schema == 1) {
    // vq4_ops.rs:193-207: every slot live, capacities in slot order, then
    // output distinct from the four inputs, status distinct from all five.
    for (int i = 0; i < n; ++i)
      if (ids[i] == 0) return PlanError::NullIdentity;
    for (int i = 0; i < n; ++i)
      if (capacities[i] < p.required[i]) {
        *slot = i;
        return PlanError::Capacity;
      }
    for (int i = 0; i < 4; ++i)
      if (ids[i] == ids[4]) return PlanError::OutputAlias;
    for (int i = 0; i < 5; ++i)
      if (ids[i] == ids[5]) return PlanError::StatusAlias;
    return PlanError::None;
  }
  // Schema 2: a slot the operation reads or writes must be live; an unused
  // slot may be null. Each written slot is distinct from every other used slot.
  for (int i = 0; i < n; ++i)
    if (p.required[i] && ids[i] == 0) return PlanError::NullIdentity;
  for (int i = 0; i < n; ++i)
    if (p.required[i] && capacities[i] < p.required[i]) {
      *slot = i;
      return PlanError::Capacity;
    }
  // written: out0, out1, and in4 for the fit (its workspace)
  for (int o = 4; o < 7; ++o) {
    if (!p.required[o] || (o == 4 && !p.writes_in4())) continue;
    for (int i = 0; i < n; ++i)
      if (i != o && p.required[i] && ids[i] == ids[o] && i != 7) return PlanError::OutputAlias;
  }
  for (int i = 0; i < 7; ++i)
    if (p.required[i] && ids[i] == ids[7]) return PlanError::StatusAlias;
  return PlanError::None;
}

PlanError validate_dispatch(const Plan& p, const std::array<uint32_t, 3>& limits) {
  for (int i = 0; i < 3; ++i)
    if (p.dispatch[i] == 0 || p.dispatch[i] > limits[i]) return PlanError::Dispatch;
  return PlanError::None;
}

std::string plan_error_name(PlanError e, int schema, int slot) {
  const char* pre = schema == 1 ? "vq-" : "vq2-";
  switch (e) {
    case PlanError::None: return "";
    case PlanError::Operation: return std::string(pre) + "operation-out-of-range";
    case PlanError::Group: return std::string(pre) + "unsupported-group";
    case PlanError::Entries: return std::string(pre) + "codebook-entries-not-16";
    case PlanError::Flags: return std::string(pre) + "unsupported-flags";
    case PlanError::Reserved: return std::string(pre) + "nonzero-reserved-word";
    case PlanError::Geometry: return std::string(pre) + "invalid-geometry";
    case PlanError::AddressLimit: return std::string(pre) + "address-limit-exceeded";
    case PlanError::WorkLimit: return std::string(pre) + "matmul-work-limit";
    case PlanError::Capacity: return std::string(pre) + "binding-" + std::to_string(slot) + "-too-small";
    case PlanError::NullIdentity: return std::string(pre) + "null-allocation-identity";
    case PlanError::OutputAlias: return std::string(pre) + "output-aliases-input";
    case PlanError::StatusAlias: return std::string(pre) + "status-aliases-operand";
    case PlanError::Dispatch: return std::string(pre) + "dispatch-grid-unsupported";
    case PlanError::Batch: return std::string(pre) + "invalid-batch";
    case PlanError::Aux: return std::string(pre) + "invalid-aux-word";
    case PlanError::Misaligned: return std::string(pre) + "operand-misaligned";
  }
  return "vq-unknown";
}

int32_t plan_error_code(PlanError e) {
  switch (e) {
    case PlanError::Capacity:
    case PlanError::AddressLimit:
    case PlanError::WorkLimit:
      return ACK_ERR_SIZE;
    default:
      return ACK_ERR_SHAPE;
  }
}

}  // namespace ack
