// Expert row-block gather for the pipelined residency engine (the address-table
// gather of experts4bit_qlora/engines/pipelined.py:117-150, rewritten as a CUDA
// kernel of this library).
//
// Each MoE layer keeps, per expert, one row-block holding its four weight segments
// (gate_up packed, gate_up absmax, down packed, down absmax) either in a resident
// device stack (hot experts) or in a pinned host arena (cold experts), and a device
// table src_table[e] = the row-block's address (device memory, or pinned host memory
// under unified addressing). The fused layer reads four device stacks
// [resident rows | slots, segment]: resident experts in place, the others from the
// slot of the pick that asked for them. A decode step asks for the k experts its
// token routed to: pick j is served from resident row resident_row[ids[j]] when that
// is >= 0, else from slot j, which is filled here unless `have[j]` already holds
// ids[j]; local_ids[j] receives the stack row the layer must read. have[j] is updated
// in a second launch (so no CTA of a slot sees the update while its peers still copy).
// Nothing depends on the ids on the host: the launch geometry is fixed, so a
// decode step built on it is capturable in a CUDA graph.
#include "common.cuh"

namespace e4b {
namespace {

struct GatherArgs {
  const uint64_t* src_table;
  int E;
  const int64_t* ids;
  const int64_t* have;
  int n;
  const int32_t* resident_row;  // [E] row in the resident stack, -1 = not resident (nullable)
  int resident_rows;            // rows before the slots in the stacks
  int64_t* local_ids;           // [n] stack row each pick reads (nullable)
  uint64_t seg_off[4];    // segment offsets inside a source row-block (bytes, 16-aligned)
  uint64_t seg_bytes[4];  // segment sizes (bytes, multiples of 16)
  char* seg_dst[4];       // stacks: slot j of segment s at seg_dst[s] + (resident_rows + j) * seg_bytes[s]
  uint64_t total;         // sum of seg_bytes
  int* err;
};

__global__ void __launch_bounds__(256) gather_rows_kernel(const GatherArgs a) {
  const int j = blockIdx.y;
  const int64_t id = a.ids[j];
  const bool lead = blockIdx.x == 0 && threadIdx.x == 0;
  if (id < 0 || id >= a.E) {
    if (lead) {
      raise_error(a.err, E4B_ERR_EXPERT_INDEX);
      if (a.local_ids) a.local_ids[j] = a.resident_rows + j;
    }
    return;
  }
  const int rr = a.resident_row ? a.resident_row[id] : -1;
  if (lead && a.local_ids) a.local_ids[j] = rr >= 0 ? rr : a.resident_rows + j;
  if (rr >= 0) return;                    // read in place from the resident stack
  if (a.have && a.have[j] == id) return;  // the slot already holds this expert
  const char* src = reinterpret_cast<const char*>(a.src_table[id]);
  const uint64_t vecs = a.total / 16;
  for (uint64_t v = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; v < vecs; v += (uint64_t)gridDim.x * blockDim.x) {
    uint64_t o = v * 16;
    int s = 0;
    while (s < 3 && o >= a.seg_bytes[s]) {
      o -= a.seg_bytes[s];
      ++s;
    }
    const uint4 val = ldg_u4(src + a.seg_off[s] + o);
    *reinterpret_cast<uint4*>(a.seg_dst[s] + (uint64_t)(a.resident_rows + j) * a.seg_bytes[s] + o) = val;
  }
}

__global__ void commit_have_kernel(const int64_t* ids, const int32_t* resident_row, int E, int64_t* have, int n) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= n) return;
  const int64_t id = ids[j];
  if (id < 0 || id >= E || (resident_row && resident_row[id] >= 0)) return;  // the slot was not written
  have[j] = id;
}

}  // namespace
}  // namespace e4b

using namespace e4b;

extern "C" e4b_status e4b_gather_expert_rows(const uint64_t* src_table, int num_experts, const int64_t* ids,
                                             int64_t* have, int slots, const int32_t* resident_row,
                                             int resident_rows, int64_t* local_ids, const uint64_t* seg_off_host,
                                             const uint64_t* seg_bytes_host, void* const* seg_dst_host, void* workspace,
                                             size_t workspace_bytes, void* stream) {
  if (!src_table || !ids || num_experts <= 0 || slots < 0 || !seg_off_host || !seg_bytes_host || !seg_dst_host)
    return E4B_ERR_INVALID_ARG;
  if (slots == 0) return E4B_OK;
  if (!workspace || workspace_bytes < kErrBytes) return E4B_ERR_WORKSPACE;
  GatherArgs a{};
  a.src_table = src_table;
  a.E = num_experts;
  a.ids = ids;
  a.have = have;
  a.n = slots;
  a.resident_row = resident_row;
  a.resident_rows = resident_rows < 0 ? 0 : resident_rows;
  a.local_ids = local_ids;
  a.total = 0;
  for (int s = 0; s < 4; ++s) {
    a.seg_off[s] = seg_off_host[s];
    a.seg_bytes[s] = seg_bytes_host[s];
    a.seg_dst[s] = static_cast<char*>(seg_dst_host[s]);
    if ((a.seg_off[s] | a.seg_bytes[s]) & 15) return E4B_ERR_ALIGNMENT;
    if (a.seg_bytes[s] && (!a.seg_dst[s] || !aligned16(a.seg_dst[s]))) return E4B_ERR_ALIGNMENT;
    a.total += a.seg_bytes[s];
  }
  a.err = static_cast<int*>(workspace);
  cudaStream_t st = (cudaStream_t)stream;
  // one CTA per 256 KB of a row-block (at most 128 per slot): enough copies in flight per slot
  int cols = (int)((a.total + (256u << 10) - 1) >> 18);
  cols = cols < 1 ? 1 : (cols > 128 ? 128 : cols);
  gather_rows_kernel<<<dim3(cols, slots), 256, 0, st>>>(a);
  if (launch_status() != E4B_OK) return E4B_ERR_CUDA;
  if (have) {
    commit_have_kernel<<<(slots + 127) / 128, 128, 0, st>>>(ids, resident_row, num_experts, have, slots);
    if (launch_status() != E4B_OK) return E4B_ERR_CUDA;
  }
  return E4B_OK;
}
