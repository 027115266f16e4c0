// JSON and binary (.cugraph v1) serialization of GraphDesc.
//
// Parity: reference csrc/CUDAGraph.cpp:1001-1502 (JSON writer),
// csrc/BinaryGraphIO.cpp:15-371 (binary writer), 379-737 (readers). The JSON
// keys follow the reference's schema so tools that read one archive can read
// the other; the binary reader here fills GraphDesc directly (no JSON
// round-trip), which is the fast path used by every LOAD.
#include <stdio.h>
#include <string.h>
#include <sys/stat.h>

#include <fstream>
#include <map>
#include <stdexcept>
#include <string>
#include <unordered_map>

#include "cugraph_format.h"
#include "graph_desc.h"

namespace fbc {
namespace J = fb::json;

namespace {

const char kHex[] = "0123456789abcdef";

std::string to_hex(const uint8_t* p, size_t n) {
  std::string s(n * 2, '0');
  for (size_t i = 0; i < n; ++i) {
    s[2 * i] = kHex[p[i] >> 4];
    s[2 * i + 1] = kHex[p[i] & 15];
  }
  return s;
}

int hexval(char c) {
  if (c >= '0' && c <= '9') return c - '0';
  if (c >= 'a' && c <= 'f') return c - 'a' + 10;
  if (c >= 'A' && c <= 'F') return c - 'A' + 10;
  throw std::runtime_error("bad hex digit in graph file");
}

std::vector<uint8_t> from_hex(const std::string& s) {
  if (s.size() % 2) throw std::runtime_error("odd-length hex string in graph file");
  std::vector<uint8_t> out(s.size() / 2);
  for (size_t i = 0; i < out.size(); ++i)
    out[i] = static_cast<uint8_t>(hexval(s[2 * i]) * 16 + hexval(s[2 * i + 1]));
  return out;
}

std::string hash_hex(uint64_t h) {
  char buf[24];
  snprintf(buf, sizeof(buf), "%016llx", static_cast<unsigned long long>(h));
  return buf;
}

J::Object attrs_to_json(const NodeAttrs& a) {
  J::Object o;
  o["attrQueryAvailable"] = static_cast<int>(a.attr_query_available);
  if (a.flags & KNA_CLUSTER_DIM) {
    o["clusterDimX"] = a.cluster[0];
    o["clusterDimY"] = a.cluster[1];
    o["clusterDimZ"] = a.cluster[2];
  }
  if (a.flags & KNA_PREFERRED_CLUSTER_DIM) {
    o["preferredClusterDimX"] = a.preferred_cluster[0];
    o["preferredClusterDimY"] = a.preferred_cluster[1];
    o["preferredClusterDimZ"] = a.preferred_cluster[2];
  }
  if (a.flags & KNA_CLUSTER_SCHEDULING) o["clusterSchedulingPolicyPreference"] = a.cluster_sched_policy;
  if (a.flags & KNA_COOPERATIVE) o["cooperative"] = a.cooperative;
  if (a.flags & KNA_PRIORITY) o["priority"] = a.priority;
  if (a.flags & KNA_MEM_SYNC_DOMAIN) o["memSyncDomain"] = a.mem_sync_domain;
  if (a.flags & KNA_MEM_SYNC_DOMAIN_MAP) {
    o["memSyncDomainMapDefault"] = static_cast<int>(a.mem_sync_map_default);
    o["memSyncDomainMapRemote"] = static_cast<int>(a.mem_sync_map_remote);
  }
  if (a.flags & KNA_SHARED_MEM_CARVEOUT) o["preferredSharedMemCarveout"] = a.preferred_carveout;
  return o;
}

NodeAttrs attrs_from_json(const J::Object& o) {
  NodeAttrs a;
  if (const J::Value* v = o.find("attrQueryAvailable")) a.attr_query_available = static_cast<uint8_t>(v->as_i64());
  if (o.contains("clusterDimX")) {
    a.flags |= KNA_CLUSTER_DIM;
    a.cluster[0] = static_cast<uint32_t>(o.at("clusterDimX").as_u64());
    a.cluster[1] = static_cast<uint32_t>(o.at("clusterDimY").as_u64());
    a.cluster[2] = static_cast<uint32_t>(o.at("clusterDimZ").as_u64());
  }
  if (o.contains("preferredClusterDimX")) {
    a.flags |= KNA_PREFERRED_CLUSTER_DIM;
    a.preferred_cluster[0] = static_cast<uint32_t>(o.at("preferredClusterDimX").as_u64());
    a.preferred_cluster[1] = static_cast<uint32_t>(o.at("preferredClusterDimY").as_u64());
    a.preferred_cluster[2] = static_cast<uint32_t>(o.at("preferredClusterDimZ").as_u64());
  }
  if (const J::Value* v = o.find("clusterSchedulingPolicyPreference")) {
    a.flags |= KNA_CLUSTER_SCHEDULING;
    a.cluster_sched_policy = static_cast<int32_t>(v->as_i64());
  }
  if (const J::Value* v = o.find("cooperative")) {
    a.flags |= KNA_COOPERATIVE;
    a.cooperative = static_cast<int32_t>(v->as_i64());
  }
  if (const J::Value* v = o.find("priority")) {
    a.flags |= KNA_PRIORITY;
    a.priority = static_cast<int32_t>(v->as_i64());
  }
  if (const J::Value* v = o.find("memSyncDomain")) {
    a.flags |= KNA_MEM_SYNC_DOMAIN;
    a.mem_sync_domain = static_cast<int32_t>(v->as_i64());
  }
  if (o.contains("memSyncDomainMapDefault")) {
    a.flags |= KNA_MEM_SYNC_DOMAIN_MAP;
    a.mem_sync_map_default = static_cast<uint8_t>(o.at("memSyncDomainMapDefault").as_i64());
    a.mem_sync_map_remote = static_cast<uint8_t>(o.at("memSyncDomainMapRemote").as_i64());
  }
  if (const J::Value* v = o.find("preferredSharedMemCarveout")) {
    a.flags |= KNA_SHARED_MEM_CARVEOUT;
    a.preferred_carveout = static_cast<uint32_t>(v->as_u64());
  }
  return a;
}

J::Object memset_to_json(const CUDA_MEMSET_NODE_PARAMS& m) {
  J::Object o;
  o["dst"] = static_cast<unsigned long long>(m.dst);
  o["elementSize"] = m.elementSize;
  o["height"] = static_cast<unsigned long long>(m.height);
  o["pitch"] = static_cast<unsigned long long>(m.pitch);
  o["value"] = m.value;
  o["width"] = static_cast<unsigned long long>(m.width);
  return o;
}

CUDA_MEMSET_NODE_PARAMS memset_from_json(const J::Object& o) {
  CUDA_MEMSET_NODE_PARAMS m;
  memset(&m, 0, sizeof(m));
  m.dst = o.at("dst").as_u64();
  m.elementSize = static_cast<unsigned>(o.at("elementSize").as_u64());
  m.height = o.at("height").as_u64();
  m.pitch = o.at("pitch").as_u64();
  m.value = static_cast<unsigned>(o.at("value").as_u64());
  m.width = o.at("width").as_u64();
  return m;
}

#define MEMCPY_FIELDS(X)                                                                  \
  X(Depth) X(Height) X(WidthInBytes) X(dstDevice) X(dstHeight) X(dstLOD) X(dstPitch)     \
      X(dstXInBytes) X(dstY) X(dstZ) X(srcDevice) X(srcHeight) X(srcLOD) X(srcPitch)      \
          X(srcXInBytes) X(srcY) X(srcZ)

J::Object memcpy_to_json(const CUDA_MEMCPY3D& m) {
  J::Object o;
#define W(f) o[#f] = static_cast<unsigned long long>(m.f);
  MEMCPY_FIELDS(W)
#undef W
  o["dstMemoryType"] = static_cast<int>(m.dstMemoryType);
  o["srcMemoryType"] = static_cast<int>(m.srcMemoryType);
  return o;
}

CUDA_MEMCPY3D memcpy_from_json(const J::Object& o) {
  CUDA_MEMCPY3D m;
  memset(&m, 0, sizeof(m));
#define R(f) m.f = static_cast<decltype(m.f)>(o.at(#f).as_u64());
  MEMCPY_FIELDS(R)
#undef R
  m.dstMemoryType = static_cast<CUmemorytype>(o.at("dstMemoryType").as_i64());
  m.srcMemoryType = static_cast<CUmemorytype>(o.at("srcMemoryType").as_i64());
  return m;
}

}  // namespace

J::Value to_json(const GraphDesc& g) {
  J::Array nodes;
  for (const Node& n : g.nodes) {
    J::Object no;
    no["id"] = n.id;
    no["type"] = node_type_name(n.type);
    J::Object p;
    switch (n.type) {
      case NodeType::Kernel: {
        const KernelNode& k = n.kernel;
        p["blockDimX"] = k.block[0];
        p["blockDimY"] = k.block[1];
        p["blockDimZ"] = k.block[2];
        p["gridDimX"] = k.grid[0];
        p["gridDimY"] = k.grid[1];
        p["gridDimZ"] = k.grid[2];
        p["sharedMemBytes"] = k.smem;
        if (k.attrs.flags) p["kernel_node_attrs"] = J::Value(attrs_to_json(k.attrs));
        if (k.has_extra) {
          p["extra"] = true;
          p["extra_argBuffer_hex"] = to_hex(k.extra_buffer.data(), k.extra_buffer.size());
        } else {
          J::Array params;
          size_t off = 0;
          for (size_t i = 0; i < k.params.size(); ++i) {
            J::Object po;
            po["index"] = static_cast<unsigned long long>(i);
            po["offset"] = static_cast<unsigned long long>(off);
            po["size"] = static_cast<unsigned long long>(k.params[i].size());
            po["value_hex"] = to_hex(k.params[i].data(), k.params[i].size());
            off += k.params[i].size();
            params.push_back(J::Value(std::move(po)));
          }
          p["kernelParams"] = J::Value(std::move(params));
        }
        p["function_name"] = k.func_name;
        p["kernel_source_binary_hash"] = hash_hex(k.binary_hash);
        J::Object fa;
        fa["max_dynamic_shared_size_bytes"] = k.max_dynamic_smem;
        fa["preferred_shared_memory_carveout"] = k.preferred_carveout;
        fa["cluster_scheduling_policy_preference"] = k.cluster_sched_pref;
        fa["required_cluster_width"] = k.required_cluster[0];
        fa["required_cluster_height"] = k.required_cluster[1];
        fa["required_cluster_depth"] = k.required_cluster[2];
        p["func_attrs"] = J::Value(std::move(fa));
        break;
      }
      case NodeType::Memset: p = memset_to_json(n.memset); break;
      case NodeType::Memcpy: p = memcpy_to_json(n.memcpy); break;
      case NodeType::EventRecord:
      case NodeType::EventWait: p["event_id"] = n.event_id; break;
      case NodeType::Empty: break;
    }
    no["params"] = J::Value(std::move(p));
    nodes.push_back(J::Value(std::move(no)));
  }
  J::Object root;
  root["nodes"] = J::Value(std::move(nodes));
  if (g.has_deps) {
    J::Array deps;
    for (size_t i = 0; i < g.deps.size(); ++i) {
      J::Object d;
      d["from"] = g.deps[i].first;
      d["to"] = g.deps[i].second;
      if (!g.edge_data.empty() && !g.edge_data[i].is_default()) {
        d["from_port"] = static_cast<int>(g.edge_data[i].from_port);
        d["to_port"] = static_cast<int>(g.edge_data[i].to_port);
        d["type"] = static_cast<int>(g.edge_data[i].type);
      }
      deps.push_back(J::Value(std::move(d)));
    }
    root["dependencies"] = J::Value(std::move(deps));
  }
  root["topology_key"] = g.topology_key;
  if (g.has_common_attrs) root["common_kernel_node_attrs"] = J::Value(attrs_to_json(g.common_attrs));
  J::Array gens;
  for (const auto& gen : g.generators) {
    J::Object o;
    o["id"] = static_cast<unsigned long long>(gen.id);
    o["seed"] = static_cast<unsigned long long>(gen.seed);
    o["wholegraph_increment"] = static_cast<unsigned long long>(gen.wholegraph_increment);
    if (gen.seed_ptr) {
      o["seed_ptr"] = static_cast<unsigned long long>(gen.seed_ptr);
      o["offset_ptr"] = static_cast<unsigned long long>(gen.offset_ptr);
    }
    gens.push_back(J::Value(std::move(o)));
  }
  root["generators"] = J::Value(std::move(gens));
  root["num_events"] = g.num_events;
  if (!g.allocator_events_json.empty()) root["allocator_events"] = J::parse(g.allocator_events_json);
  if (!g.output_tensors_json.empty()) root["output_tensors"] = J::parse(g.output_tensors_json);
  return J::Value(std::move(root));
}

std::shared_ptr<GraphDesc> from_json(const J::Value& v) {
  auto g = std::make_shared<GraphDesc>();
  const J::Object& root = v.as_object();
  for (const J::Value& nv : root.at("nodes").as_array()) {
    const J::Object& no = nv.as_object();
    Node n;
    n.id = static_cast<uint32_t>(no.at("id").as_u64());
    if (!node_type_from_name(no.at("type").as_string(), &n.type))
      throw std::runtime_error("unknown node type '" + no.at("type").as_string() + "'");
    const J::Object& p = no.at("params").as_object();
    switch (n.type) {
      case NodeType::Kernel: {
        KernelNode& k = n.kernel;
        k.block[0] = static_cast<uint32_t>(p.at("blockDimX").as_u64());
        k.block[1] = static_cast<uint32_t>(p.at("blockDimY").as_u64());
        k.block[2] = static_cast<uint32_t>(p.at("blockDimZ").as_u64());
        k.grid[0] = static_cast<uint32_t>(p.at("gridDimX").as_u64());
        k.grid[1] = static_cast<uint32_t>(p.at("gridDimY").as_u64());
        k.grid[2] = static_cast<uint32_t>(p.at("gridDimZ").as_u64());
        k.smem = static_cast<uint32_t>(p.at("sharedMemBytes").as_u64());
        if (const J::Value* a = p.find("kernel_node_attrs")) k.attrs = attrs_from_json(a->as_object());
        if (const J::Value* e = p.find("extra"); e && e->as_bool()) {
          k.has_extra = true;
          k.extra_buffer = from_hex(p.at("extra_argBuffer_hex").as_string());
        } else if (const J::Value* kp = p.find("kernelParams")) {
          for (const J::Value& pv : kp->as_array())
            k.params.push_back(from_hex(pv.as_object().at("value_hex").as_string()));
        }
        k.func_name = p.at("function_name").as_string();
        k.binary_hash = strtoull(p.at("kernel_source_binary_hash").as_string().c_str(), nullptr, 16);
        if (const J::Value* fav = p.find("func_attrs")) {
          const J::Object& fa = fav->as_object();
          k.max_dynamic_smem = static_cast<int32_t>(fa.at("max_dynamic_shared_size_bytes").as_i64());
          k.preferred_carveout = static_cast<int32_t>(fa.at("preferred_shared_memory_carveout").as_i64());
          k.cluster_sched_pref = static_cast<int32_t>(fa.at("cluster_scheduling_policy_preference").as_i64());
          k.required_cluster[0] = static_cast<int32_t>(fa.at("required_cluster_width").as_i64());
          k.required_cluster[1] = static_cast<int32_t>(fa.at("required_cluster_height").as_i64());
          k.required_cluster[2] = static_cast<int32_t>(fa.at("required_cluster_depth").as_i64());
        }
        break;
      }
      case NodeType::Memset: n.memset = memset_from_json(p); break;
      case NodeType::Memcpy: n.memcpy = memcpy_from_json(p); break;
      case NodeType::EventRecord:
      case NodeType::EventWait: n.event_id = static_cast<int32_t>(p.at("event_id").as_i64()); break;
      case NodeType::Empty: break;
    }
    g->nodes.push_back(std::move(n));
  }
  if (const J::Value* deps = root.find("dependencies")) {
    bool plain = true;
    for (const J::Value& dv : deps->as_array()) {
      const J::Object& o = dv.as_object();
      g->deps.emplace_back(static_cast<uint32_t>(o.at("from").as_u64()), static_cast<uint32_t>(o.at("to").as_u64()));
      EdgeData e;
      if (const J::Value* v = o.find("from_port")) e.from_port = static_cast<uint8_t>(v->as_u64());
      if (const J::Value* v = o.find("to_port")) e.to_port = static_cast<uint8_t>(v->as_u64());
      if (const J::Value* v = o.find("type")) e.type = static_cast<uint8_t>(v->as_u64());
      g->edge_data.push_back(e);
      plain = plain && e.is_default();
    }
    if (plain) g->edge_data.clear();
  } else {
    g->has_deps = false;
  }
  g->topology_key = root.at("topology_key").as_string();
  if (const J::Value* ca = root.find("common_kernel_node_attrs")) {
    g->has_common_attrs = true;
    g->common_attrs = attrs_from_json(ca->as_object());
  }
  if (const J::Value* gens = root.find("generators"))
    for (const J::Value& gv : gens->as_array()) {
      const J::Object& o = gv.as_object();
      Generator gen{o.at("id").as_u64(), o.at("seed").as_u64(), o.at("wholegraph_increment").as_u64()};
      if (const J::Value* sp = o.find("seed_ptr")) gen.seed_ptr = sp->as_u64();
      if (const J::Value* op = o.find("offset_ptr")) gen.offset_ptr = op->as_u64();
      g->generators.push_back(gen);
    }
  if (const J::Value* ne = root.find("num_events")) g->num_events = static_cast<int>(ne->as_i64());
  if (const J::Value* ae = root.find("allocator_events")) g->allocator_events_json = ae->dump();
  if (const J::Value* ot = root.find("output_tensors")) g->output_tensors_json = ot->dump();
  return g;
}

// ---- binary ---------------------------------------------------------------------

namespace {

void attrs_to_rec(const NodeAttrs& a, bin::KernelRec* r) {
  r->kna_flags = a.flags;
  memcpy(r->cluster, a.cluster, sizeof(r->cluster));
  memcpy(r->preferred_cluster, a.preferred_cluster, sizeof(r->preferred_cluster));
  r->cluster_sched_policy = a.cluster_sched_policy;
  r->cooperative = a.cooperative;
  r->priority = a.priority;
  r->mem_sync_domain = a.mem_sync_domain;
  r->mem_sync_map_default = a.mem_sync_map_default;
  r->mem_sync_map_remote = a.mem_sync_map_remote;
  r->attr_query_available = a.attr_query_available;
  r->preferred_smem_carveout = a.preferred_carveout;
}

NodeAttrs attrs_from_rec(const bin::KernelRec& r) {
  NodeAttrs a;
  a.flags = r.kna_flags;
  memcpy(a.cluster, r.cluster, sizeof(a.cluster));
  memcpy(a.preferred_cluster, r.preferred_cluster, sizeof(a.preferred_cluster));
  a.cluster_sched_policy = r.cluster_sched_policy;
  a.cooperative = r.cooperative;
  a.priority = r.priority;
  a.mem_sync_domain = r.mem_sync_domain;
  a.mem_sync_map_default = r.mem_sync_map_default;
  a.mem_sync_map_remote = r.mem_sync_map_remote;
  a.attr_query_available = r.attr_query_available;
  a.preferred_carveout = r.preferred_smem_carveout;
  return a;
}

struct StringTable {
  std::string data;
  std::unordered_map<std::string, uint32_t> offsets;
  uint32_t count = 0;
  uint32_t add(const std::string& s) {
    auto it = offsets.find(s);
    if (it != offsets.end()) return it->second;
    uint32_t off = static_cast<uint32_t>(data.size());
    data += s;
    data.push_back('\0');
    offsets[s] = off;
    ++count;
    return off;
  }
};

}  // namespace

void write_binary(const GraphDesc& g, const std::string& path) {
  StringTable strings;
  std::vector<bin::NodeRec> nodes(g.nodes.size());
  std::vector<bin::ParamRec> pindex;
  std::string pdata, argbuf;
  for (size_t i = 0; i < g.nodes.size(); ++i) {
    const Node& n = g.nodes[i];
    bin::NodeRec& r = nodes[i];
    memset(&r, 0, sizeof(r));
    r.node_id = n.id;
    r.type = static_cast<uint8_t>(n.type);
    switch (n.type) {
      case NodeType::Kernel: {
        const KernelNode& k = n.kernel;
        bin::KernelRec& kr = r.kernel;
        memcpy(kr.block, k.block, sizeof(kr.block));
        memcpy(kr.grid, k.grid, sizeof(kr.grid));
        kr.smem = k.smem;
        kr.binary_hash = k.binary_hash;
        kr.name_off = strings.add(k.func_name);
        kr.name_len = static_cast<uint32_t>(k.func_name.size());
        kr.max_dynamic_smem = k.max_dynamic_smem;
        kr.preferred_carveout = k.preferred_carveout;
        kr.cluster_sched_pref = k.cluster_sched_pref;
        memcpy(kr.required_cluster, k.required_cluster, sizeof(kr.required_cluster));
        attrs_to_rec(k.attrs, &kr);
        kr.param_index_off = static_cast<uint32_t>(pindex.size() * sizeof(bin::ParamRec));
        kr.num_params = static_cast<uint32_t>(k.params.size());
        for (const auto& p : k.params) {
          pindex.push_back(bin::ParamRec{static_cast<uint32_t>(pdata.size()),
                                         static_cast<uint32_t>(p.size())});
          pdata.append(reinterpret_cast<const char*>(p.data()), p.size());
        }
        if (k.has_extra) {
          kr.arg_buffer_off = static_cast<uint32_t>(argbuf.size());
          kr.arg_buffer_size = static_cast<uint32_t>(k.extra_buffer.size());
          argbuf.append(reinterpret_cast<const char*>(k.extra_buffer.data()), k.extra_buffer.size());
        } else {
          kr.arg_buffer_off = 0xFFFFFFFFu;
        }
        break;
      }
      case NodeType::Memset: {
        const auto& m = n.memset;
        r.memset.dst = m.dst;
        r.memset.element_size = m.elementSize;
        r.memset.height = m.height;
        r.memset.pitch = m.pitch;
        r.memset.value = m.value;
        r.memset.width = m.width;
        break;
      }
      case NodeType::Memcpy: {
        const auto& m = n.memcpy;
        auto& c = r.memcpy;
        c.depth = m.Depth;
        c.height = m.Height;
        c.width_bytes = m.WidthInBytes;
        c.dst_device = m.dstDevice;
        c.dst_height = m.dstHeight;
        c.dst_lod = m.dstLOD;
        c.dst_pitch = m.dstPitch;
        c.dst_x_bytes = m.dstXInBytes;
        c.dst_y = m.dstY;
        c.dst_z = m.dstZ;
        c.dst_memory_type = m.dstMemoryType;
        c.src_device = m.srcDevice;
        c.src_height = m.srcHeight;
        c.src_lod = m.srcLOD;
        c.src_pitch = m.srcPitch;
        c.src_x_bytes = m.srcXInBytes;
        c.src_y = m.srcY;
        c.src_z = m.srcZ;
        c.src_memory_type = m.srcMemoryType;
        break;
      }
      case NodeType::EventRecord:
      case NodeType::EventWait: r.event.event_id = n.event_id; break;
      case NodeType::Empty: break;
    }
  }
  const bool edge_data = !g.edge_data.empty();
  std::vector<bin::DepRec> deps;
  std::vector<bin::DepDataRec> deps_d;
  for (size_t i = 0; i < g.deps.size(); ++i) {
    if (edge_data) {
      const EdgeData& e = g.edge_data.at(i);
      deps_d.push_back(bin::DepDataRec{g.deps[i].first, g.deps[i].second, e.from_port, e.to_port, e.type, 0});
    } else {
      deps.push_back(bin::DepRec{g.deps[i].first, g.deps[i].second});
    }
  }
  bin::CommonAttrsRec common;
  memset(&common, 0, sizeof(common));
  if (g.has_common_attrs) {
    bin::KernelRec tmp;
    memset(&tmp, 0, sizeof(tmp));
    attrs_to_rec(g.common_attrs, &tmp);
    common.flags = tmp.kna_flags;
    memcpy(common.cluster, tmp.cluster, sizeof(common.cluster));
    memcpy(common.preferred_cluster, tmp.preferred_cluster, sizeof(common.preferred_cluster));
    common.cluster_sched_policy = tmp.cluster_sched_policy;
    common.cooperative = tmp.cooperative;
    common.priority = tmp.priority;
    common.mem_sync_domain = tmp.mem_sync_domain;
    common.mem_sync_map_default = tmp.mem_sync_map_default;
    common.mem_sync_map_remote = tmp.mem_sync_map_remote;
    common.attr_query_available = tmp.attr_query_available;
    common.preferred_smem_carveout = tmp.preferred_smem_carveout;
  }
  bool gen_ptrs = false;
  for (const auto& gen : g.generators) gen_ptrs = gen_ptrs || gen.seed_ptr != 0;
  std::vector<bin::GeneratorRec> gens;
  std::vector<bin::GeneratorPtrRec> gens_p;
  for (const auto& gen : g.generators) {
    const bin::GeneratorRec r{gen.id, gen.seed, gen.wholegraph_increment};
    if (gen_ptrs)
      gens_p.push_back(bin::GeneratorPtrRec{r, gen.seed_ptr, gen.offset_ptr});
    else
      gens.push_back(r);
  }

  // Assemble sections.
  struct Blob {
    const void* p;
    size_t n;
  };
  Blob blobs[bin::S_COUNT] = {
      {strings.data.data(), strings.data.size()},
      {nodes.data(), nodes.size() * sizeof(bin::NodeRec)},
      {edge_data ? static_cast<const void*>(deps_d.data()) : static_cast<const void*>(deps.data()),
       edge_data ? deps_d.size() * sizeof(bin::DepDataRec) : deps.size() * sizeof(bin::DepRec)},
      {pindex.data(), pindex.size() * sizeof(bin::ParamRec)},
      {pdata.data(), pdata.size()},
      {argbuf.data(), argbuf.size()},
      {&common, g.has_common_attrs ? sizeof(common) : 0},
      {gen_ptrs ? static_cast<const void*>(gens_p.data()) : static_cast<const void*>(gens.data()),
       gen_ptrs ? gens_p.size() * sizeof(bin::GeneratorPtrRec) : gens.size() * sizeof(bin::GeneratorRec)},
      {g.allocator_events_json.data(), g.allocator_events_json.size()},
      {g.output_tensors_json.data(), g.output_tensors_json.size()},
      {g.topology_key.data(), g.topology_key.size()},
  };
  bin::Header h;
  memset(&h, 0, sizeof(h));
  memcpy(h.magic, bin::kMagic, 8);
  h.version = bin::kVersion;
  h.flags = (g.has_common_attrs ? bin::HF_COMMON_ATTRS : 0) | (g.has_deps ? bin::HF_DEPS : 0) |
            (!g.allocator_events_json.empty() ? bin::HF_ALLOC_EVENTS : 0) |
            (!g.output_tensors_json.empty() ? bin::HF_OUTPUTS : 0) |
            (!g.generators.empty() ? bin::HF_GENERATORS : 0) | (gen_ptrs ? bin::HF_GENERATOR_PTRS : 0) |
            (edge_data ? bin::HF_EDGE_DATA : 0);
  h.num_nodes = static_cast<uint32_t>(nodes.size());
  h.num_deps = static_cast<uint32_t>(g.deps.size());
  h.num_generators = static_cast<uint32_t>(g.generators.size());
  h.num_sections = bin::S_COUNT;
  h.num_strings = strings.count;
  // num_events has no header field in v1; it is stored in the reserved bytes.
  uint32_t ne = static_cast<uint32_t>(g.num_events);
  memcpy(h.reserved, &ne, sizeof(ne));

  std::string out;
  out.append(reinterpret_cast<const char*>(&h), sizeof(h));
  bin::SectionEntry dir[bin::S_COUNT];
  uint64_t off = sizeof(h) + sizeof(dir);
  for (uint32_t s = 0; s < bin::S_COUNT; ++s) {
    off = (off + 7) & ~7ull;
    dir[s] = bin::SectionEntry{s, 0, off, blobs[s].n};
    off += blobs[s].n;
  }
  out.append(reinterpret_cast<const char*>(dir), sizeof(dir));
  for (uint32_t s = 0; s < bin::S_COUNT; ++s) {
    out.resize(dir[s].offset, '\0');
    out.append(static_cast<const char*>(blobs[s].p), blobs[s].n);
  }
  std::string tmp = path + ".tmp";
  {
    std::ofstream f(tmp, std::ios::binary | std::ios::trunc);
    if (!f) throw std::runtime_error("cannot write " + tmp);
    f.write(out.data(), static_cast<std::streamsize>(out.size()));
    if (!f) throw std::runtime_error("short write to " + tmp);
  }
  if (rename(tmp.c_str(), path.c_str()) != 0) throw std::runtime_error("cannot rename " + tmp);
}

std::shared_ptr<GraphDesc> read_binary(const std::string& path) {
  std::ifstream f(path, std::ios::binary | std::ios::ate);
  if (!f) return nullptr;
  std::streamsize size = f.tellg();
  f.seekg(0);
  std::vector<uint8_t> data(static_cast<size_t>(size));
  if (size && !f.read(reinterpret_cast<char*>(data.data()), size))
    throw std::runtime_error("cannot read " + path);
  auto fail = [&](const char* why) { throw std::runtime_error(path + ": corrupt .cugraph (" + why + ")"); };
  if (data.size() < sizeof(bin::Header) + bin::S_COUNT * sizeof(bin::SectionEntry)) fail("too short");
  bin::Header h;
  memcpy(&h, data.data(), sizeof(h));
  if (memcmp(h.magic, bin::kMagic, 8) != 0) fail("bad magic");
  if (h.version != bin::kVersion) fail("unsupported version");
  if (h.num_sections < bin::S_COUNT) fail("missing sections");
  const bin::SectionEntry* dir = reinterpret_cast<const bin::SectionEntry*>(data.data() + sizeof(h));
  for (uint32_t s = 0; s < bin::S_COUNT; ++s)
    if (dir[s].offset + dir[s].size > data.size()) fail("section out of bounds");
  auto sec = [&](uint32_t s) { return data.data() + dir[s].offset; };
  auto g = std::make_shared<GraphDesc>();
  if (dir[bin::S_NODES].size != h.num_nodes * sizeof(bin::NodeRec)) fail("node table size");
  const char* strings = reinterpret_cast<const char*>(sec(bin::S_STRINGS));
  const size_t strings_size = dir[bin::S_STRINGS].size;
  const uint8_t* pindex = sec(bin::S_PARAM_INDEX);
  const size_t pindex_size = dir[bin::S_PARAM_INDEX].size;
  const uint8_t* pdata = sec(bin::S_PARAM_DATA);
  const size_t pdata_size = dir[bin::S_PARAM_DATA].size;
  const uint8_t* args = sec(bin::S_ARG_BUFFERS);
  const size_t args_size = dir[bin::S_ARG_BUFFERS].size;
  g->nodes.resize(h.num_nodes);
  for (uint32_t i = 0; i < h.num_nodes; ++i) {
    bin::NodeRec r;
    memcpy(&r, sec(bin::S_NODES) + i * sizeof(bin::NodeRec), sizeof(r));
    Node& n = g->nodes[i];
    n.id = r.node_id;
    if (r.type > static_cast<uint8_t>(NodeType::Empty)) fail("bad node type");
    n.type = static_cast<NodeType>(r.type);
    switch (n.type) {
      case NodeType::Kernel: {
        const bin::KernelRec& kr = r.kernel;
        KernelNode& k = n.kernel;
        memcpy(k.block, kr.block, sizeof(k.block));
        memcpy(k.grid, kr.grid, sizeof(k.grid));
        k.smem = kr.smem;
        k.binary_hash = kr.binary_hash;
        if (static_cast<size_t>(kr.name_off) + kr.name_len > strings_size) fail("name out of bounds");
        k.func_name.assign(strings + kr.name_off, kr.name_len);
        k.max_dynamic_smem = kr.max_dynamic_smem;
        k.preferred_carveout = kr.preferred_carveout;
        k.cluster_sched_pref = kr.cluster_sched_pref;
        memcpy(k.required_cluster, kr.required_cluster, sizeof(k.required_cluster));
        k.attrs = attrs_from_rec(kr);
        if (static_cast<size_t>(kr.param_index_off) + kr.num_params * sizeof(bin::ParamRec) > pindex_size)
          fail("param index out of bounds");
        k.params.resize(kr.num_params);
        for (uint32_t p = 0; p < kr.num_params; ++p) {
          bin::ParamRec pr;
          memcpy(&pr, pindex + kr.param_index_off + p * sizeof(bin::ParamRec), sizeof(pr));
          if (static_cast<size_t>(pr.data_off) + pr.size > pdata_size) fail("param data out of bounds");
          k.params[p].assign(pdata + pr.data_off, pdata + pr.data_off + pr.size);
        }
        if (kr.arg_buffer_off != 0xFFFFFFFFu) {
          if (static_cast<size_t>(kr.arg_buffer_off) + kr.arg_buffer_size > args_size) fail("arg buffer out of bounds");
          k.has_extra = true;
          k.extra_buffer.assign(args + kr.arg_buffer_off, args + kr.arg_buffer_off + kr.arg_buffer_size);
        }
        break;
      }
      case NodeType::Memset: {
        auto& m = n.memset;
        m.dst = r.memset.dst;
        m.elementSize = r.memset.element_size;
        m.height = r.memset.height;
        m.pitch = r.memset.pitch;
        m.value = r.memset.value;
        m.width = r.memset.width;
        break;
      }
      case NodeType::Memcpy: {
        auto& m = n.memcpy;
        const auto& c = r.memcpy;
        m.Depth = c.depth;
        m.Height = c.height;
        m.WidthInBytes = c.width_bytes;
        m.dstDevice = c.dst_device;
        m.dstHeight = c.dst_height;
        m.dstLOD = c.dst_lod;
        m.dstPitch = c.dst_pitch;
        m.dstXInBytes = c.dst_x_bytes;
        m.dstY = c.dst_y;
        m.dstZ = c.dst_z;
        m.dstMemoryType = static_cast<CUmemorytype>(c.dst_memory_type);
        m.srcDevice = c.src_device;
        m.srcHeight = c.src_height;
        m.srcLOD = c.src_lod;
        m.srcPitch = c.src_pitch;
        m.srcXInBytes = c.src_x_bytes;
        m.srcY = c.src_y;
        m.srcZ = c.src_z;
        m.srcMemoryType = static_cast<CUmemorytype>(c.src_memory_type);
        break;
      }
      case NodeType::EventRecord:
      case NodeType::EventWait: n.event_id = r.event.event_id; break;
      case NodeType::Empty: break;
    }
  }
  g->has_deps = (h.flags & bin::HF_DEPS) != 0;
  const bool edge_data = (h.flags & bin::HF_EDGE_DATA) != 0;
  const size_t dep_rec = edge_data ? sizeof(bin::DepDataRec) : sizeof(bin::DepRec);
  if (dir[bin::S_DEPS].size != h.num_deps * dep_rec) fail("dependency table size");
  for (uint32_t i = 0; i < h.num_deps; ++i) {
    bin::DepDataRec d{};
    memcpy(&d, sec(bin::S_DEPS) + i * dep_rec, dep_rec);
    g->deps.emplace_back(d.from, d.to);
    if (edge_data) g->edge_data.push_back(EdgeData{d.from_port, d.to_port, d.type});
  }
  if (h.flags & bin::HF_COMMON_ATTRS) {
    if (dir[bin::S_COMMON_ATTRS].size < sizeof(bin::CommonAttrsRec)) fail("common attrs size");
    bin::CommonAttrsRec c;
    memcpy(&c, sec(bin::S_COMMON_ATTRS), sizeof(c));
    g->has_common_attrs = true;
    NodeAttrs& a = g->common_attrs;
    a.flags = c.flags;
    memcpy(a.cluster, c.cluster, sizeof(a.cluster));
    memcpy(a.preferred_cluster, c.preferred_cluster, sizeof(a.preferred_cluster));
    a.cluster_sched_policy = c.cluster_sched_policy;
    a.cooperative = c.cooperative;
    a.priority = c.priority;
    a.mem_sync_domain = c.mem_sync_domain;
    a.mem_sync_map_default = c.mem_sync_map_default;
    a.mem_sync_map_remote = c.mem_sync_map_remote;
    a.attr_query_available = c.attr_query_available;
    a.preferred_carveout = c.preferred_smem_carveout;
  }
  const bool gen_ptrs = (h.flags & bin::HF_GENERATOR_PTRS) != 0;
  const size_t gen_rec = gen_ptrs ? sizeof(bin::GeneratorPtrRec) : sizeof(bin::GeneratorRec);
  if (dir[bin::S_GENERATORS].size != h.num_generators * gen_rec) fail("generator table size");
  for (uint32_t i = 0; i < h.num_generators; ++i) {
    bin::GeneratorPtrRec r{};
    memcpy(&r, sec(bin::S_GENERATORS) + i * gen_rec, gen_rec);
    g->generators.push_back(
        Generator{r.base.id, r.base.seed, r.base.wholegraph_increment, r.seed_ptr, r.offset_ptr});
  }
  g->allocator_events_json.assign(reinterpret_cast<const char*>(sec(bin::S_ALLOC_EVENTS)),
                                  dir[bin::S_ALLOC_EVENTS].size);
  g->output_tensors_json.assign(reinterpret_cast<const char*>(sec(bin::S_OUTPUTS)),
                                dir[bin::S_OUTPUTS].size);
  g->topology_key.assign(reinterpret_cast<const char*>(sec(bin::S_TOPOLOGY)), dir[bin::S_TOPOLOGY].size);
  uint32_t ne = 0;
  memcpy(&ne, h.reserved, sizeof(ne));
  g->num_events = static_cast<int>(ne);
  return g;
}

std::string cugraph_path_for(const std::string& json_path) {
  const std::string ext = ".json";
  if (json_path.size() > ext.size() &&
      json_path.compare(json_path.size() - ext.size(), ext.size(), ext) == 0)
    return json_path.substr(0, json_path.size() - ext.size()) + ".cugraph";
  return json_path + ".cugraph";
}

std::shared_ptr<GraphDesc> read_graph_file(const std::string& json_path) {
  auto g = read_binary(cugraph_path_for(json_path));
  if (g) return g;
  std::ifstream f(json_path, std::ios::binary);
  if (!f) throw std::runtime_error("graph file not found: " + json_path);
  std::string text((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
  return from_json(J::parse(text));
}

}  // namespace fbc
