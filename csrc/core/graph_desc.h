// In-memory description of a persisted CUDA graph and the operations on it:
// analysis of a live CUgraph, JSON and binary (.cugraph v1) serialization,
// and rebuilding a CUgraph/CUgraphExec from the description.
//
// Parity: reference include/metadata.h:10-215 (node metadata),
// csrc/CUDAGraph.cpp:630-941 (analysis), 1001-1502 (JSON save),
// csrc/BinaryGraphIO.cpp (binary I/O), csrc/CUDAGraphParallel.cpp:171-834
// (building from parsed data).
#pragma once

#include <cuda.h>

#include <array>
#include <cstdint>
#include <memory>
#include <string>
#include <vector>

#include "../common/fb_json.h"

namespace fbc {

enum class NodeType : uint8_t { Kernel = 0, Memset = 1, Memcpy = 2, EventRecord = 3, EventWait = 4, Empty = 5 };

const char* node_type_name(NodeType t);  // "KernelNode", ...
bool node_type_from_name(const std::string& s, NodeType* out);

// Kernel-node launch attributes worth persisting (non-default values only).
struct NodeAttrs {
  uint32_t flags = 0;  // KNA_* bits below
  uint32_t cluster[3] = {0, 0, 0};
  uint32_t preferred_cluster[3] = {0, 0, 0};
  int32_t cluster_sched_policy = 0;
  int32_t cooperative = 0;
  int32_t priority = 0;
  int32_t mem_sync_domain = 0;
  uint8_t mem_sync_map_default = 0;
  uint8_t mem_sync_map_remote = 0;
  uint8_t attr_query_available = 0;
  uint32_t preferred_carveout = 0;
  bool operator==(const NodeAttrs& o) const;
};
enum : uint32_t {
  KNA_CLUSTER_DIM = 1u << 0,
  KNA_PREFERRED_CLUSTER_DIM = 1u << 1,
  KNA_CLUSTER_SCHEDULING = 1u << 2,
  KNA_COOPERATIVE = 1u << 3,
  KNA_PRIORITY = 1u << 4,
  KNA_MEM_SYNC_DOMAIN = 1u << 5,
  KNA_MEM_SYNC_DOMAIN_MAP = 1u << 6,
  KNA_SHARED_MEM_CARVEOUT = 1u << 7,
  KNA_ATTR_QUERY_AVAILABLE = 1u << 8,
};

struct KernelNode {
  uint32_t grid[3] = {1, 1, 1};
  uint32_t block[3] = {1, 1, 1};
  uint32_t smem = 0;
  uint64_t binary_hash = 0;
  std::string func_name;
  // Function attributes to re-apply on LOAD.
  int32_t max_dynamic_smem = 0;
  int32_t preferred_carveout = -1;
  int32_t cluster_sched_pref = 0;
  int32_t required_cluster[3] = {0, 0, 0};
  NodeAttrs attrs;
  // Arguments: either per-parameter bytes, or one packed "extra" buffer.
  std::vector<std::vector<uint8_t>> params;
  bool has_extra = false;
  std::vector<uint8_t> extra_buffer;
  // Live handles (capture process, or after resolution on LOAD).
  CUfunction func = nullptr;
};

struct Node {
  uint32_t id = 0;
  NodeType type = NodeType::Empty;
  KernelNode kernel;
  CUDA_MEMSET_NODE_PARAMS memset{};
  CUDA_MEMCPY3D memcpy{};
  int32_t event_id = -1;
};

// A random-number generator whose state the graph's kernels read. The
// kernels hold the device addresses of the generator's graph seed and offset
// words (seed_ptr, offset_ptr; 0 when unknown); before every replay the host
// writes the generator's seed and current offset there and advances the
// offset by wholegraph_increment.
struct Generator {
  uint64_t id = 0, seed = 0, wholegraph_increment = 0;
  uint64_t seed_ptr = 0, offset_ptr = 0;
};

// Data of one dependency edge (CUgraphEdgeData): all zero for a plain
// full-completion dependency; programmatic dependent launch edges set the
// ports and type.
struct EdgeData {
  uint8_t from_port = 0, to_port = 0, type = 0;
  bool is_default() const { return from_port == 0 && to_port == 0 && type == 0; }
  bool operator==(const EdgeData& o) const {
    return from_port == o.from_port && to_port == o.to_port && type == o.type;
  }
};

struct GraphDesc {
  std::vector<Node> nodes;
  std::vector<std::pair<uint32_t, uint32_t>> deps;  // (from, to) node ids
  std::vector<EdgeData> edge_data;  // parallel to deps; empty when every edge is a plain dependency
  bool has_deps = true;     // false for on-demand members stripped by the manifest
  std::string topology_key;
  bool has_common_attrs = false;
  NodeAttrs common_attrs;   // shared by every kernel node (hoisted)
  std::vector<Generator> generators;
  std::string allocator_events_json;  // {"start_base_addr":..,"events":[..]} or ""
  std::string output_tensors_json;    // JSON text produced by the Python layer or ""
  int num_events = 0;
};

// ---- analysis of a live graph ------------------------------------------------
// Walks every node; kernel nodes are identified through the module registry.
// Throws std::runtime_error with a clear message on unsupported content.
std::shared_ptr<GraphDesc> analyze_graph(CUgraph graph);

// Topology key: node type sequence + cluster dims per kernel + edge-list hash.
std::string compute_topology_key(const GraphDesc& g);
// Hoist launch attributes shared by all kernel nodes into common_attrs.
void hoist_common_attrs(GraphDesc& g);

// ---- serialization -------------------------------------------------------------
fb::json::Value to_json(const GraphDesc& g);
std::shared_ptr<GraphDesc> from_json(const fb::json::Value& v);
void write_binary(const GraphDesc& g, const std::string& path);
// Returns null if the file is absent; throws on a corrupt file.
std::shared_ptr<GraphDesc> read_binary(const std::string& path);
// Reads X.cugraph next to X.json when present, else X.json.
std::shared_ptr<GraphDesc> read_graph_file(const std::string& json_path);
std::string cugraph_path_for(const std::string& json_path);

// ---- rebuilding ------------------------------------------------------------------
// Resolves every kernel node's function through the registry (and applies
// function attributes), fills KernelNode::func.
void resolve_functions(GraphDesc& g);

struct BuiltGraph {
  CUgraph graph = nullptr;
  std::vector<CUgraphNode> nodes;   // index = node position in GraphDesc::nodes
  std::vector<CUevent> events;      // created for event nodes
  ~BuiltGraph();
};
std::unique_ptr<BuiltGraph> build_graph(const GraphDesc& g);
CUgraphExec instantiate(CUgraph graph);

// Fills CUDA_KERNEL_NODE_PARAMS for node k; ptrs must outlive the call.
void make_kernel_params(const KernelNode& k, CUDA_KERNEL_NODE_PARAMS* p, std::vector<void*>* ptrs,
                        std::vector<void*>* extra);

bool kernel_launch_equal(const KernelNode& a, const KernelNode& b);

// Moves the generators' seed/offset words to seed_slot / seed_slot + 8: every
// 8-byte-aligned word of a kernel parameter (or packed argument buffer) that
// equals a generator's seed_ptr or offset_ptr is rewritten, and the generator
// records take the new addresses. Returns the number of words rewritten.
size_t relocate_generator_words(GraphDesc& g, uint64_t seed_slot);

void check_drv(CUresult r, const char* what);

}  // namespace fbc
