// Analysis of live CUDA graphs and rebuilding graphs from a GraphDesc.
//
// Parity: reference csrc/CUDAGraph.cpp:630-941 (analyze_captured_graph),
// 1338-1441 (topology key, common attrs), CUDAGraph.cpp:1506-2098 and
// CUDAGraphParallel.cpp:171-834 (graph building). Our own implementation:
// one code path builds every graph (template or stand-alone), kernel
// functions are always resolved through the registry by (hash, name), and
// every failure is an exception carrying the driver status, never an abort.
#include <stdio.h>
#include <string.h>

#include <map>
#include <stdexcept>
#include <string>
#include <unordered_map>

#include "../common/fb_crc64.h"
#include "../common/fb_driver.h"
#include "../common/fb_hook_api.h"
#include "graph_desc.h"

namespace fbc {

void check_drv(CUresult r, const char* what) {
  if (r == CUDA_SUCCESS) return;
  const char* name = nullptr;
  if (fb_driver()->cuGetErrorName) fb_driver()->cuGetErrorName(r, &name);
  throw std::runtime_error(std::string(what) + " failed: " + (name ? name : "?") + " (" +
                           std::to_string(static_cast<int>(r)) + ")");
}

const char* node_type_name(NodeType t) {
  switch (t) {
    case NodeType::Kernel: return "KernelNode";
    case NodeType::Memset: return "MemsetNode";
    case NodeType::Memcpy: return "MemcpyNode";
    case NodeType::EventRecord: return "EventRecordNode";
    case NodeType::EventWait: return "EventWaitNode";
    case NodeType::Empty: return "EmptyNode";
  }
  return "?";
}

bool node_type_from_name(const std::string& s, NodeType* out) {
  static const std::map<std::string, NodeType> m = {
      {"KernelNode", NodeType::Kernel},         {"MemsetNode", NodeType::Memset},
      {"MemcpyNode", NodeType::Memcpy},         {"EventRecordNode", NodeType::EventRecord},
      {"EventWaitNode", NodeType::EventWait},   {"EmptyNode", NodeType::Empty}};
  auto it = m.find(s);
  if (it == m.end()) return false;
  *out = it->second;
  return true;
}

bool NodeAttrs::operator==(const NodeAttrs& o) const {
  return flags == o.flags && memcmp(cluster, o.cluster, sizeof(cluster)) == 0 &&
         memcmp(preferred_cluster, o.preferred_cluster, sizeof(preferred_cluster)) == 0 &&
         cluster_sched_policy == o.cluster_sched_policy && cooperative == o.cooperative &&
         priority == o.priority && mem_sync_domain == o.mem_sync_domain &&
         mem_sync_map_default == o.mem_sync_map_default &&
         mem_sync_map_remote == o.mem_sync_map_remote &&
         attr_query_available == o.attr_query_available &&
         preferred_carveout == o.preferred_carveout;
}

namespace {

void read_node_attrs(CUgraphNode n, NodeAttrs* a) {
  const FbDriver* d = fb_driver();
  if (!d->cuGraphKernelNodeGetAttribute) return;
  CUkernelNodeAttrValue v;
  auto get = [&](CUkernelNodeAttrID id) {
    memset(&v, 0, sizeof(v));
    return d->cuGraphKernelNodeGetAttribute(n, id, &v) == CUDA_SUCCESS;
  };
  if (get(CU_LAUNCH_ATTRIBUTE_CLUSTER_DIMENSION) &&
      (v.clusterDim.x > 1 || v.clusterDim.y > 1 || v.clusterDim.z > 1)) {
    a->flags |= KNA_CLUSTER_DIM;
    a->cluster[0] = v.clusterDim.x;
    a->cluster[1] = v.clusterDim.y;
    a->cluster[2] = v.clusterDim.z;
  }
  if (get(CU_LAUNCH_ATTRIBUTE_PREFERRED_CLUSTER_DIMENSION) &&
      (v.preferredClusterDim.x || v.preferredClusterDim.y || v.preferredClusterDim.z)) {
    a->flags |= KNA_PREFERRED_CLUSTER_DIM;
    a->preferred_cluster[0] = v.preferredClusterDim.x;
    a->preferred_cluster[1] = v.preferredClusterDim.y;
    a->preferred_cluster[2] = v.preferredClusterDim.z;
  }
  if (get(CU_LAUNCH_ATTRIBUTE_CLUSTER_SCHEDULING_POLICY_PREFERENCE) &&
      v.clusterSchedulingPolicyPreference != 0) {
    a->flags |= KNA_CLUSTER_SCHEDULING;
    a->cluster_sched_policy = v.clusterSchedulingPolicyPreference;
  }
  if (get(CU_LAUNCH_ATTRIBUTE_COOPERATIVE) && v.cooperative) {
    a->flags |= KNA_COOPERATIVE;
    a->cooperative = v.cooperative;
  }
  if (get(CU_LAUNCH_ATTRIBUTE_PRIORITY) && v.priority) {
    a->flags |= KNA_PRIORITY;
    a->priority = v.priority;
  }
  if (get(CU_LAUNCH_ATTRIBUTE_MEM_SYNC_DOMAIN) && v.memSyncDomain) {
    a->flags |= KNA_MEM_SYNC_DOMAIN;
    a->mem_sync_domain = v.memSyncDomain;
  }
  if (get(CU_LAUNCH_ATTRIBUTE_MEM_SYNC_DOMAIN_MAP) &&
      (v.memSyncDomainMap.default_ || v.memSyncDomainMap.remote)) {
    a->flags |= KNA_MEM_SYNC_DOMAIN_MAP;
    a->mem_sync_map_default = v.memSyncDomainMap.default_;
    a->mem_sync_map_remote = v.memSyncDomainMap.remote;
  }
  if (get(CU_LAUNCH_ATTRIBUTE_PREFERRED_SHARED_MEMORY_CARVEOUT) && v.sharedMemCarveout) {
    a->flags |= KNA_SHARED_MEM_CARVEOUT;
    a->preferred_carveout = v.sharedMemCarveout;
  }
}

void apply_node_attrs(CUgraphNode n, const NodeAttrs& a) {
  const FbDriver* d = fb_driver();
  CUkernelNodeAttrValue v;
  auto set = [&](CUkernelNodeAttrID id, const char* what) {
    check_drv(d->cuGraphKernelNodeSetAttribute(n, id, &v), what);
  };
  if (a.flags & KNA_CLUSTER_DIM) {
    memset(&v, 0, sizeof(v));
    v.clusterDim.x = a.cluster[0];
    v.clusterDim.y = a.cluster[1];
    v.clusterDim.z = a.cluster[2];
    set(CU_LAUNCH_ATTRIBUTE_CLUSTER_DIMENSION, "set cluster dim");
  }
  if (a.flags & KNA_PREFERRED_CLUSTER_DIM) {
    memset(&v, 0, sizeof(v));
    v.preferredClusterDim.x = a.preferred_cluster[0];
    v.preferredClusterDim.y = a.preferred_cluster[1];
    v.preferredClusterDim.z = a.preferred_cluster[2];
    set(CU_LAUNCH_ATTRIBUTE_PREFERRED_CLUSTER_DIMENSION, "set preferred cluster dim");
  }
  if (a.flags & KNA_CLUSTER_SCHEDULING) {
    memset(&v, 0, sizeof(v));
    v.clusterSchedulingPolicyPreference =
        static_cast<CUclusterSchedulingPolicy>(a.cluster_sched_policy);
    set(CU_LAUNCH_ATTRIBUTE_CLUSTER_SCHEDULING_POLICY_PREFERENCE, "set cluster scheduling");
  }
  if (a.flags & KNA_COOPERATIVE) {
    memset(&v, 0, sizeof(v));
    v.cooperative = a.cooperative;
    set(CU_LAUNCH_ATTRIBUTE_COOPERATIVE, "set cooperative");
  }
  if (a.flags & KNA_PRIORITY) {
    memset(&v, 0, sizeof(v));
    v.priority = a.priority;
    set(CU_LAUNCH_ATTRIBUTE_PRIORITY, "set priority");
  }
  if (a.flags & KNA_MEM_SYNC_DOMAIN) {
    memset(&v, 0, sizeof(v));
    v.memSyncDomain = static_cast<CUlaunchMemSyncDomain>(a.mem_sync_domain);
    set(CU_LAUNCH_ATTRIBUTE_MEM_SYNC_DOMAIN, "set mem sync domain");
  }
  if (a.flags & KNA_MEM_SYNC_DOMAIN_MAP) {
    memset(&v, 0, sizeof(v));
    v.memSyncDomainMap.default_ = a.mem_sync_map_default;
    v.memSyncDomainMap.remote = a.mem_sync_map_remote;
    set(CU_LAUNCH_ATTRIBUTE_MEM_SYNC_DOMAIN_MAP, "set mem sync domain map");
  }
  if (a.flags & KNA_SHARED_MEM_CARVEOUT) {
    memset(&v, 0, sizeof(v));
    v.sharedMemCarveout = a.preferred_carveout;
    set(CU_LAUNCH_ATTRIBUTE_PREFERRED_SHARED_MEMORY_CARVEOUT, "set carveout");
  }
}

void analyze_kernel(CUgraphNode n, KernelNode* k) {
  const FbDriver* d = fb_driver();
  CUDA_KERNEL_NODE_PARAMS p;
  memset(&p, 0, sizeof(p));
  check_drv(d->cuGraphKernelNodeGetParams(n, &p), "cuGraphKernelNodeGetParams");
  k->grid[0] = p.gridDimX;
  k->grid[1] = p.gridDimY;
  k->grid[2] = p.gridDimZ;
  k->block[0] = p.blockDimX;
  k->block[1] = p.blockDimY;
  k->block[2] = p.blockDimZ;
  k->smem = p.sharedMemBytes;
  CUfunction f = p.func;
  if (!f && p.kern) check_drv(d->cuKernelGetFunction(&f, p.kern), "cuKernelGetFunction");
  k->func = f;
  char name[1024];
  uint64_t hash = 0;
  if (fb_registry_identify(f, &hash, name, sizeof(name)) != FB_OK)
    throw std::runtime_error(fb_last_error());
  k->binary_hash = hash;
  k->func_name = name;
  fb_registry_mark_used(hash);
  // Parameters: sizes from the function's parameter layout.
  if (p.kernelParams) {
    for (size_t i = 0;; ++i) {
      size_t off = 0, sz = 0;
      CUresult rc = d->cuFuncGetParamInfo(f, i, &off, &sz);
      if (rc == CUDA_ERROR_INVALID_VALUE) break;
      check_drv(rc, "cuFuncGetParamInfo");
      const uint8_t* src = static_cast<const uint8_t*>(p.kernelParams[i]);
      k->params.emplace_back(src, src + sz);
    }
  } else if (p.extra) {
    void* buf = nullptr;
    size_t size = 0;
    for (int i = 0; p.extra[i] != CU_LAUNCH_PARAM_END; i += 2) {
      if (p.extra[i] == CU_LAUNCH_PARAM_BUFFER_POINTER) buf = p.extra[i + 1];
      if (p.extra[i] == CU_LAUNCH_PARAM_BUFFER_SIZE) size = *static_cast<size_t*>(p.extra[i + 1]);
    }
    k->has_extra = true;
    if (buf && size)
      k->extra_buffer.assign(static_cast<uint8_t*>(buf), static_cast<uint8_t*>(buf) + size);
  }
  // Function attributes that LOAD has to re-apply.
  int v = 0;
  if (d->cuFuncGetAttribute(&v, CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES, f) == CUDA_SUCCESS)
    k->max_dynamic_smem = v;
  if (d->cuFuncGetAttribute(&v, CU_FUNC_ATTRIBUTE_PREFERRED_SHARED_MEMORY_CARVEOUT, f) ==
      CUDA_SUCCESS)
    k->preferred_carveout = v;
  if (d->cuFuncGetAttribute(&v, CU_FUNC_ATTRIBUTE_CLUSTER_SCHEDULING_POLICY_PREFERENCE, f) ==
      CUDA_SUCCESS)
    k->cluster_sched_pref = v;
  if (d->cuFuncGetAttribute(&v, CU_FUNC_ATTRIBUTE_REQUIRED_CLUSTER_WIDTH, f) == CUDA_SUCCESS)
    k->required_cluster[0] = v;
  if (d->cuFuncGetAttribute(&v, CU_FUNC_ATTRIBUTE_REQUIRED_CLUSTER_HEIGHT, f) == CUDA_SUCCESS)
    k->required_cluster[1] = v;
  if (d->cuFuncGetAttribute(&v, CU_FUNC_ATTRIBUTE_REQUIRED_CLUSTER_DEPTH, f) == CUDA_SUCCESS)
    k->required_cluster[2] = v;
  read_node_attrs(n, &k->attrs);
}

}  // namespace

std::shared_ptr<GraphDesc> analyze_graph(CUgraph graph) {
  const FbDriver* d = fb_driver();
  auto g = std::make_shared<GraphDesc>();
  size_t n = 0;
  check_drv(d->cuGraphGetNodes(graph, nullptr, &n), "cuGraphGetNodes");
  std::vector<CUgraphNode> nodes(n);
  if (n) check_drv(d->cuGraphGetNodes(graph, nodes.data(), &n), "cuGraphGetNodes");
  std::unordered_map<CUgraphNode, uint32_t> index;
  std::unordered_map<CUevent, int> event_ids;
  g->nodes.resize(n);
  for (size_t i = 0; i < n; ++i) {
    index[nodes[i]] = static_cast<uint32_t>(i);
    Node& node = g->nodes[i];
    node.id = static_cast<uint32_t>(i);
    CUgraphNodeType t;
    check_drv(d->cuGraphNodeGetType(nodes[i], &t), "cuGraphNodeGetType");
    switch (t) {
      case CU_GRAPH_NODE_TYPE_KERNEL:
        node.type = NodeType::Kernel;
        analyze_kernel(nodes[i], &node.kernel);
        break;
      case CU_GRAPH_NODE_TYPE_MEMSET:
        node.type = NodeType::Memset;
        check_drv(d->cuGraphMemsetNodeGetParams(nodes[i], &node.memset), "memset params");
        break;
      case CU_GRAPH_NODE_TYPE_MEMCPY: {
        node.type = NodeType::Memcpy;
        check_drv(d->cuGraphMemcpyNodeGetParams(nodes[i], &node.memcpy), "memcpy params");
        const auto& m = node.memcpy;
        if (m.srcMemoryType != CU_MEMORYTYPE_DEVICE || m.dstMemoryType != CU_MEMORYTYPE_DEVICE)
          throw std::runtime_error(
              "graph contains a memcpy node touching host memory; only device-to-device "
              "copies can be persisted (host addresses do not survive the process)");
        break;
      }
      case CU_GRAPH_NODE_TYPE_EVENT_RECORD:
      case CU_GRAPH_NODE_TYPE_WAIT_EVENT: {
        node.type = t == CU_GRAPH_NODE_TYPE_EVENT_RECORD ? NodeType::EventRecord
                                                         : NodeType::EventWait;
        CUevent e = nullptr;
        check_drv(t == CU_GRAPH_NODE_TYPE_EVENT_RECORD
                      ? d->cuGraphEventRecordNodeGetEvent(nodes[i], &e)
                      : d->cuGraphEventWaitNodeGetEvent(nodes[i], &e),
                  "event node");
        auto it = event_ids.find(e);
        if (it == event_ids.end()) it = event_ids.emplace(e, static_cast<int>(event_ids.size())).first;
        node.event_id = it->second;
        break;
      }
      case CU_GRAPH_NODE_TYPE_EMPTY: node.type = NodeType::Empty; break;
      default:
        throw std::runtime_error("graph node type " + std::to_string(static_cast<int>(t)) +
                                 " cannot be persisted (kernel, memset, device memcpy, event "
                                 "and empty nodes are supported)");
    }
  }
  g->num_events = static_cast<int>(event_ids.size());
  size_t ne = 0;
  if (d->cuGraphGetEdges_v2) {
    // Edge data (ports, type) as well: graphs with programmatic dependent
    // launch edges cannot be described by the plain query (it reports
    // CUDA_ERROR_LOSSY_QUERY for them).
    check_drv(d->cuGraphGetEdges_v2(graph, nullptr, nullptr, nullptr, &ne), "cuGraphGetEdges_v2");
    if (ne) {
      std::vector<CUgraphNode> from(ne), to(ne);
      std::vector<CUgraphEdgeData> data(ne);
      check_drv(d->cuGraphGetEdges_v2(graph, from.data(), to.data(), data.data(), &ne), "cuGraphGetEdges_v2");
      bool plain = true;
      for (size_t i = 0; i < ne; ++i) {
        g->deps.emplace_back(index.at(from[i]), index.at(to[i]));
        g->edge_data.push_back(EdgeData{data[i].from_port, data[i].to_port, data[i].type});
        plain = plain && g->edge_data.back().is_default();
      }
      if (plain) g->edge_data.clear();
    }
  } else {
    check_drv(d->cuGraphGetEdges(graph, nullptr, nullptr, &ne), "cuGraphGetEdges");
    if (ne) {
      std::vector<CUgraphNode> from(ne), to(ne);
      check_drv(d->cuGraphGetEdges(graph, from.data(), to.data(), &ne), "cuGraphGetEdges");
      for (size_t i = 0; i < ne; ++i) g->deps.emplace_back(index.at(from[i]), index.at(to[i]));
    }
  }
  g->topology_key = compute_topology_key(*g);
  hoist_common_attrs(*g);
  return g;
}

std::string compute_topology_key(const GraphDesc& g) {
  std::string key;
  key.reserve(g.nodes.size() * 14 + 24);
  for (size_t i = 0; i < g.nodes.size(); ++i) {
    if (i) key += ',';
    const Node& n = g.nodes[i];
    key += node_type_name(n.type);
    if (n.type == NodeType::Kernel) {
      const KernelNode& k = n.kernel;
      uint32_t cx = 0, cy = 0, cz = 0;
      const NodeAttrs& a = (k.attrs.flags & KNA_CLUSTER_DIM) ? k.attrs : g.common_attrs;
      if (a.flags & KNA_CLUSTER_DIM) {
        cx = a.cluster[0];
        cy = a.cluster[1];
        cz = a.cluster[2];
      } else if (k.required_cluster[0] > 0) {
        cx = k.required_cluster[0];
        cy = k.required_cluster[1];
        cz = k.required_cluster[2];
      }
      if (cx || cy || cz)
        key += ":C" + std::to_string(cx) + "_" + std::to_string(cy) + "_" + std::to_string(cz);
      else
        key += ":0";
    }
  }
  // Edge structure must match too for exec updates to apply.
  if (g.has_deps) {
    uint64_t h = ~0ull;
    for (size_t i = 0; i < g.deps.size(); ++i) {
      uint32_t v[2] = {g.deps[i].first, g.deps[i].second};
      h = fb::crc64_update(h, v, sizeof(v));
      if (!g.edge_data.empty() && !g.edge_data[i].is_default()) {
        const EdgeData& e = g.edge_data[i];
        const uint8_t w[3] = {e.from_port, e.to_port, e.type};
        h = fb::crc64_update(h, w, sizeof(w));
      }
    }
    char buf[32];
    snprintf(buf, sizeof(buf), "|E%zu:%016llx", g.deps.size(), static_cast<unsigned long long>(~h));
    key += buf;
  }
  return key;
}

void hoist_common_attrs(GraphDesc& g) {
  const NodeAttrs* first = nullptr;
  for (const Node& n : g.nodes) {
    if (n.type != NodeType::Kernel) continue;
    if (!first) {
      first = &n.kernel.attrs;
      continue;
    }
    if (!(n.kernel.attrs == *first)) return;
  }
  if (!first || first->flags == 0) return;
  g.has_common_attrs = true;
  g.common_attrs = *first;
  for (Node& n : g.nodes)
    if (n.type == NodeType::Kernel) n.kernel.attrs = NodeAttrs();
}

void resolve_functions(GraphDesc& g) {
  const FbDriver* d = fb_driver();
  // Many nodes share a function; resolve each (hash, name) once.
  std::map<std::pair<uint64_t, std::string>, CUfunction> cache;
  for (Node& n : g.nodes) {
    if (n.type != NodeType::Kernel) continue;
    KernelNode& k = n.kernel;
    auto key = std::make_pair(k.binary_hash, k.func_name);
    auto it = cache.find(key);
    if (it != cache.end()) {
      k.func = it->second;
      continue;
    }
    CUfunction f = nullptr;
    if (fb_registry_function(k.binary_hash, k.func_name.c_str(), &f, nullptr) != FB_OK)
      throw std::runtime_error(fb_last_error());
    if (k.max_dynamic_smem > 0)
      check_drv(d->cuFuncSetAttribute(f, CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES,
                                      k.max_dynamic_smem),
                "cuFuncSetAttribute(max dynamic smem)");
    if (k.preferred_carveout >= 0)
      d->cuFuncSetAttribute(f, CU_FUNC_ATTRIBUTE_PREFERRED_SHARED_MEMORY_CARVEOUT,
                            k.preferred_carveout);
    cache[key] = f;
    k.func = f;
  }
}

void make_kernel_params(const KernelNode& k, CUDA_KERNEL_NODE_PARAMS* p, std::vector<void*>* ptrs,
                        std::vector<void*>* extra) {
  memset(p, 0, sizeof(*p));
  p->func = k.func;
  p->gridDimX = k.grid[0];
  p->gridDimY = k.grid[1];
  p->gridDimZ = k.grid[2];
  p->blockDimX = k.block[0];
  p->blockDimY = k.block[1];
  p->blockDimZ = k.block[2];
  p->sharedMemBytes = k.smem;
  if (k.has_extra) {
    static thread_local size_t size_slot;
    size_slot = k.extra_buffer.size();
    extra->assign({CU_LAUNCH_PARAM_BUFFER_POINTER, const_cast<uint8_t*>(k.extra_buffer.data()),
                   CU_LAUNCH_PARAM_BUFFER_SIZE, &size_slot, CU_LAUNCH_PARAM_END});
    p->extra = extra->data();
  } else {
    ptrs->clear();
    for (const auto& b : k.params) ptrs->push_back(const_cast<uint8_t*>(b.data()));
    p->kernelParams = ptrs->data();
  }
}

bool kernel_launch_equal(const KernelNode& a, const KernelNode& b) {
  return a.func == b.func && memcmp(a.grid, b.grid, sizeof(a.grid)) == 0 &&
         memcmp(a.block, b.block, sizeof(a.block)) == 0 && a.smem == b.smem &&
         a.params == b.params && a.has_extra == b.has_extra && a.extra_buffer == b.extra_buffer;
}

namespace {

size_t rewrite_words(std::vector<uint8_t>& bytes, uint64_t from_seed, uint64_t from_off, uint64_t to_seed,
                     uint64_t to_off) {
  size_t n = 0;
  for (size_t o = 0; o + 8 <= bytes.size(); o += 8) {
    uint64_t w;
    memcpy(&w, bytes.data() + o, 8);
    const uint64_t to = w == from_seed ? to_seed : w == from_off ? to_off : 0;
    if (to) {
      memcpy(bytes.data() + o, &to, 8);
      ++n;
    }
  }
  return n;
}

}  // namespace

size_t relocate_generator_words(GraphDesc& g, uint64_t seed_slot) {
  size_t n = 0;
  for (Generator& gen : g.generators) {
    if (!gen.seed_ptr || !gen.offset_ptr) continue;
    const uint64_t to_seed = seed_slot, to_off = seed_slot + 8;
    if (gen.seed_ptr == to_seed && gen.offset_ptr == to_off) continue;
    for (Node& node : g.nodes) {
      if (node.type != NodeType::Kernel) continue;
      KernelNode& k = node.kernel;
      for (auto& p : k.params) n += rewrite_words(p, gen.seed_ptr, gen.offset_ptr, to_seed, to_off);
      if (k.has_extra) n += rewrite_words(k.extra_buffer, gen.seed_ptr, gen.offset_ptr, to_seed, to_off);
    }
    gen.seed_ptr = to_seed;
    gen.offset_ptr = to_off;
  }
  return n;
}

BuiltGraph::~BuiltGraph() {
  const FbDriver* d = fb_driver();
  if (graph && d->cuGraphDestroy) d->cuGraphDestroy(graph);
  for (CUevent e : events)
    if (e && d->cuEventDestroy) d->cuEventDestroy(e);
}

std::unique_ptr<BuiltGraph> build_graph(const GraphDesc& g) {
  const FbDriver* d = fb_driver();
  std::unique_ptr<BuiltGraph> b(new BuiltGraph());
  check_drv(d->cuGraphCreate(&b->graph, 0), "cuGraphCreate");
  b->events.assign(static_cast<size_t>(g.num_events), nullptr);
  for (int i = 0; i < g.num_events; ++i)
    check_drv(d->cuEventCreate(&b->events[i], CU_EVENT_DISABLE_TIMING), "cuEventCreate");
  b->nodes.resize(g.nodes.size());
  std::vector<void*> ptrs, extra;
  for (size_t i = 0; i < g.nodes.size(); ++i) {
    const Node& n = g.nodes[i];
    CUgraphNode out = nullptr;
    switch (n.type) {
      case NodeType::Kernel: {
        CUDA_KERNEL_NODE_PARAMS p;
        make_kernel_params(n.kernel, &p, &ptrs, &extra);
        check_drv(d->cuGraphAddKernelNode(&out, b->graph, nullptr, 0, &p), "cuGraphAddKernelNode");
        const NodeAttrs& a = n.kernel.attrs.flags ? n.kernel.attrs : g.common_attrs;
        if (a.flags) apply_node_attrs(out, a);
        break;
      }
      case NodeType::Memset: {
        CUcontext ctx = nullptr;
        d->cuCtxGetCurrent(&ctx);
        check_drv(d->cuGraphAddMemsetNode(&out, b->graph, nullptr, 0, &n.memset, ctx),
                  "cuGraphAddMemsetNode");
        break;
      }
      case NodeType::Memcpy: {
        CUcontext ctx = nullptr;
        d->cuCtxGetCurrent(&ctx);
        check_drv(d->cuGraphAddMemcpyNode(&out, b->graph, nullptr, 0, &n.memcpy, ctx),
                  "cuGraphAddMemcpyNode");
        break;
      }
      case NodeType::EventRecord:
        check_drv(d->cuGraphAddEventRecordNode(&out, b->graph, nullptr, 0, b->events.at(n.event_id)),
                  "cuGraphAddEventRecordNode");
        break;
      case NodeType::EventWait:
        check_drv(d->cuGraphAddEventWaitNode(&out, b->graph, nullptr, 0, b->events.at(n.event_id)),
                  "cuGraphAddEventWaitNode");
        break;
      case NodeType::Empty:
        check_drv(d->cuGraphAddEmptyNode(&out, b->graph, nullptr, 0), "cuGraphAddEmptyNode");
        break;
    }
    b->nodes[i] = out;
  }
  if (!g.has_deps && g.nodes.size() > 1)
    throw std::runtime_error("graph has no dependency table (an on-demand member cannot be built "
                             "stand-alone)");
  if (!g.deps.empty()) {
    std::vector<CUgraphNode> from, to;
    from.reserve(g.deps.size());
    to.reserve(g.deps.size());
    for (const auto& e : g.deps) {
      if (e.first >= b->nodes.size() || e.second >= b->nodes.size())
        throw std::runtime_error("dependency references a node id out of range");
      from.push_back(b->nodes[e.first]);
      to.push_back(b->nodes[e.second]);
    }
    if (!g.edge_data.empty()) {
      if (g.edge_data.size() != g.deps.size()) throw std::runtime_error("edge data does not match the edge list");
      if (!d->cuGraphAddDependencies_v2)
        throw std::runtime_error("graph has programmatic dependency edges; this driver cannot add them");
      std::vector<CUgraphEdgeData> data(g.edge_data.size());
      for (size_t i = 0; i < data.size(); ++i) {
        memset(&data[i], 0, sizeof(data[i]));
        data[i].from_port = g.edge_data[i].from_port;
        data[i].to_port = g.edge_data[i].to_port;
        data[i].type = g.edge_data[i].type;
      }
      check_drv(d->cuGraphAddDependencies_v2(b->graph, from.data(), to.data(), data.data(), from.size()),
                "cuGraphAddDependencies_v2");
    } else {
      check_drv(d->cuGraphAddDependencies(b->graph, from.data(), to.data(), from.size()),
                "cuGraphAddDependencies");
    }
  }
  return b;
}

CUgraphExec instantiate(CUgraph graph) {
  CUgraphExec exec = nullptr;
  check_drv(fb_driver()->cuGraphInstantiate(&exec, graph, 0), "cuGraphInstantiate");
  return exec;
}

}  // namespace fbc
