// Restore engine: templates, on-demand members, and the two-phase parallel
// loader. See restore.h for the design.
#include "restore.h"

#include <string.h>
#include <sys/stat.h>

#include <algorithm>
#include <chrono>
#include <fstream>
#include <map>
#include <stdexcept>
#include <unordered_map>

#include "../common/fb_driver.h"
#include "../common/fb_hook_api.h"

namespace fbc {

namespace {

double ms_since(std::chrono::steady_clock::time_point t0) {
  return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
}

uint64_t now_ns() {
  return static_cast<uint64_t>(
      std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now().time_since_epoch())
          .count());
}

bool memset_equal(const CUDA_MEMSET_NODE_PARAMS& a, const CUDA_MEMSET_NODE_PARAMS& b) {
  return a.dst == b.dst && a.pitch == b.pitch && a.value == b.value && a.elementSize == b.elementSize &&
         a.width == b.width && a.height == b.height;
}

bool memcpy_equal(const CUDA_MEMCPY3D& a, const CUDA_MEMCPY3D& b) {
  return memcmp(&a, &b, sizeof(a)) == 0;
}

// Write node `pos` of `src` into `exec` (whose graph nodes are `built`).
void patch_node(CUgraphExec exec, const BuiltGraph& built, const GraphDesc& src, uint32_t pos) {
  const FbDriver* d = fb_driver();
  const Node& n = src.nodes[pos];
  CUgraphNode gn = built.nodes.at(pos);
  switch (n.type) {
    case NodeType::Kernel: {
      CUDA_KERNEL_NODE_PARAMS p;
      std::vector<void*> ptrs, extra;
      make_kernel_params(n.kernel, &p, &ptrs, &extra);
      check_drv(d->cuGraphExecKernelNodeSetParams(exec, gn, &p), "cuGraphExecKernelNodeSetParams");
      break;
    }
    case NodeType::Memset: {
      CUcontext ctx = nullptr;
      d->cuCtxGetCurrent(&ctx);
      check_drv(d->cuGraphExecMemsetNodeSetParams(exec, gn, &n.memset, ctx),
                "cuGraphExecMemsetNodeSetParams");
      break;
    }
    case NodeType::Memcpy: {
      CUcontext ctx = nullptr;
      d->cuCtxGetCurrent(&ctx);
      check_drv(d->cuGraphExecMemcpyNodeSetParams(exec, gn, &n.memcpy, ctx),
                "cuGraphExecMemcpyNodeSetParams");
      break;
    }
    default: break;
  }
}

}  // namespace

SharedExec::~SharedExec() {
  if (exec && fb_driver()->cuGraphExecDestroy) fb_driver()->cuGraphExecDestroy(exec);
}

RestoredGraph::~RestoredGraph() {
  CUgraphExec e = own_exec.load(std::memory_order_acquire);
  if (e && fb_driver()->cuGraphExecDestroy) fb_driver()->cuGraphExecDestroy(e);
  if (shared) {
    std::lock_guard<std::mutex> lk(shared->mu);
    if (shared->current == this) shared->current = nullptr;
  }
}

std::vector<uint32_t> diff_against(const GraphDesc& tmpl, const GraphDesc& member) {
  if (tmpl.nodes.size() != member.nodes.size())
    throw std::runtime_error("topology group member has a different node count than its template");
  std::vector<uint32_t> out;
  for (uint32_t i = 0; i < tmpl.nodes.size(); ++i) {
    const Node& a = tmpl.nodes[i];
    const Node& b = member.nodes[i];
    if (a.type != b.type) throw std::runtime_error("topology group member differs in node types");
    bool differs = false;
    switch (a.type) {
      case NodeType::Kernel: differs = !kernel_launch_equal(a.kernel, b.kernel); break;
      case NodeType::Memset: differs = !memset_equal(a.memset, b.memset); break;
      case NodeType::Memcpy: differs = !memcpy_equal(a.memcpy, b.memcpy); break;
      default: break;
    }
    if (differs) out.push_back(i);
  }
  return out;
}

void RestoredGraph::launch(CUstream stream) {
  const FbDriver* d = fb_driver();
  if (CUgraphExec e = own_exec.load(std::memory_order_acquire)) {
    check_drv(d->cuGraphLaunch(e, stream), "cuGraphLaunch");
    return;
  }
  if (!shared || !shared->exec) throw std::runtime_error("graph has no executable (load failed?)");
  std::lock_guard<std::mutex> lk(shared->mu);
  if (shared->current != this) {
    const uint64_t t0 = now_ns();
    // Nodes that the previously loaded member changed must be set back, and
    // nodes this member changes must be set: patch the union with our values.
    std::vector<uint32_t> todo = diff_nodes;
    if (shared->current) {
      todo.insert(todo.end(), shared->current->diff_nodes.begin(), shared->current->diff_nodes.end());
      std::sort(todo.begin(), todo.end());
      todo.erase(std::unique(todo.begin(), todo.end()), todo.end());
    } else if (!is_template) {
      // Unknown state (e.g. after a member was destroyed): patch every node.
      todo.clear();
      for (uint32_t i = 0; i < desc->nodes.size(); ++i) todo.push_back(i);
    }
    for (uint32_t pos : todo) patch_node(shared->exec, *shared->built, *desc, pos);
    shared->current = this;
    shared->switches++;
    last_switch_ns = now_ns() - t0;
  }
  check_drv(d->cuGraphLaunch(shared->exec, stream), "cuGraphLaunch");
}

void RestoredGraph::materialize() {
  std::lock_guard<std::mutex> lk(materialize_mu);
  if (own_exec.load(std::memory_order_acquire)) return;
  if (ctx) check_drv(fb_driver()->cuCtxSetCurrent(ctx), "cuCtxSetCurrent");
  GraphDesc g = *desc;
  if (!g.has_deps && shared && shared->template_desc) {
    g.deps = shared->template_desc->deps;
    g.edge_data = shared->template_desc->edge_data;
    g.has_deps = true;
  }
  own_built = build_graph(g);
  own_exec.store(instantiate(own_built->graph), std::memory_order_release);
}

std::shared_ptr<RestoredGraph> restore_single(std::shared_ptr<GraphDesc> desc, const std::string& path) {
  resolve_functions(*desc);
  auto shared = std::make_shared<SharedExec>();
  shared->template_desc = desc;
  shared->built = build_graph(*desc);
  shared->exec = instantiate(shared->built->graph);
  auto r = std::make_shared<RestoredGraph>();
  r->desc = desc;
  r->shared = shared;
  r->path = path;
  r->is_template = true;
  fb_driver()->cuCtxGetCurrent(&r->ctx);
  shared->current = r.get();
  return r;
}

// ---- parallel loader -------------------------------------------------------------

namespace {

std::string dirname_of(const std::string& p) {
  auto s = p.find_last_of('/');
  return s == std::string::npos ? "." : p.substr(0, s);
}
std::string basename_of(const std::string& p) {
  auto s = p.find_last_of('/');
  return s == std::string::npos ? p : p.substr(s + 1);
}

template <typename F>
void parallel_for(size_t n, int threads, F&& f) {
  if (n == 0) return;
  threads = std::max(1, std::min<int>(threads, static_cast<int>(n)));
  std::atomic<size_t> next{0};
  std::exception_ptr err;
  std::mutex err_mu;
  auto body = [&]() {
    for (;;) {
      size_t i = next.fetch_add(1);
      if (i >= n) return;
      try {
        f(i);
      } catch (...) {
        std::lock_guard<std::mutex> lk(err_mu);
        if (!err) err = std::current_exception();
      }
    }
  };
  std::vector<std::thread> pool;
  for (int t = 1; t < threads; ++t) pool.emplace_back(body);
  body();
  for (auto& th : pool) th.join();
  if (err) std::rethrow_exception(err);
}

}  // namespace

std::shared_ptr<PendingLoads> start_graph_builds(const std::vector<std::string>& paths, int num_threads,
                                                 uint64_t rng_slot) {
  auto pl = std::make_shared<PendingLoads>();
  pl->paths = paths;
  pl->num_threads = num_threads;
  fb_driver()->cuCtxGetCurrent(&pl->ctx);
  const auto t0 = std::chrono::steady_clock::now();
  // Phase 1: read every graph file in parallel (binary fast path).
  pl->descs.resize(paths.size());
  parallel_for(paths.size(), num_threads, [&](size_t i) {
    pl->descs[i] = read_graph_file(paths[i]);
    if (rng_slot) relocate_generator_words(*pl->descs[i], rng_slot);
  });
  // Grouping: the manifest when present, else topology keys in file order.
  std::map<std::string, int> by_name;
  for (size_t i = 0; i < paths.size(); ++i) by_name[basename_of(paths[i])] = static_cast<int>(i);
  pl->group_of.assign(paths.size(), -1);
  const std::string manifest = paths.empty() ? "" : dirname_of(paths[0]) + "/graph_manifest.json";
  std::ifstream mf(manifest);
  if (mf) {
    std::string text((std::istreambuf_iterator<char>(mf)), std::istreambuf_iterator<char>());
    fb::json::Value m = fb::json::parse(text);
    for (const auto& gv : m.as_object().at("topology_groups").as_array()) {
      const auto& go = gv.as_object();
      int gid = -1;
      auto tit = by_name.find(go.at("template").as_string());
      for (const auto& mv : go.at("members").as_array()) {
        auto it = by_name.find(mv.as_string());
        if (it == by_name.end()) continue;
        if (gid < 0) {
          gid = static_cast<int>(pl->group_template.size());
          int tmpl = tit != by_name.end() ? tit->second : it->second;
          pl->group_template.push_back(tmpl);
          pl->group_of[tmpl] = gid;
        }
        pl->group_of[it->second] = gid;
      }
    }
  }
  std::map<std::string, int> by_key;
  for (size_t i = 0; i < paths.size(); ++i) {
    if (pl->group_of[i] >= 0) continue;
    const std::string& key = pl->descs[i]->topology_key;
    auto it = by_key.find(key);
    if (it == by_key.end()) {
      int gid = static_cast<int>(pl->group_template.size());
      pl->group_template.push_back(static_cast<int>(i));
      by_key[key] = gid;
      pl->group_of[i] = gid;
    } else {
      pl->group_of[i] = it->second;
    }
  }
  pl->groups.resize(pl->group_template.size());
  pl->diffs.resize(paths.size());
  pl->results.resize(paths.size());
  pl->finished.assign(paths.size(), 0);
  pl->resolved.assign(paths.size(), 0);
  pl->diff_ready.assign(paths.size(), 0);
  pl->deferred_reason.assign(paths.size(), std::string());
  pl->phase1_ms = ms_since(t0);
  pl->start_phase2();
  return pl;
}

void PendingLoads::start_phase2() {
  worker_ = std::thread([this]() {
    const auto t0 = std::chrono::steady_clock::now();
    try {
      const FbDriver* d = fb_driver();
      if (ctx) d->cuCtxSetCurrent(ctx);
      // Resolve functions (driver lookups, cached per image) for every graph;
      // a kernel persisted by entry name whose library has not loaded it yet
      // defers that graph to finish_one.
      for (size_t i = 0; i < descs.size(); ++i) {
        try {
          resolve_functions(*descs[i]);
          resolved[i] = 1;
        } catch (const std::exception& e) {
          deferred_reason[i] = e.what();
        }
      }
      // Templates: build + instantiate, one per group (resolved ones only).
      for (size_t gi = 0; gi < group_template.size(); ++gi) {
        if (!resolved[group_template[gi]]) continue;
        const auto& tdesc = descs[group_template[gi]];
        auto se = std::make_shared<SharedExec>();
        se->template_desc = tdesc;
        se->built = build_graph(*tdesc);
        se->exec = instantiate(se->built->graph);
        groups[gi] = se;
      }
      // On-demand members: CPU-only diffs, in parallel.
      parallel_for(descs.size(), num_threads, [&](size_t i) {
        const int tmpl = group_template[group_of[i]];
        if (static_cast<size_t>(tmpl) == i) return;
        // Exec patching only rewrites node parameters: a member must have its
        // template's node types, edges and cluster shapes, which is what the
        // topology key encodes. A manifest that groups it otherwise is stale.
        if (descs[i]->topology_key != descs[tmpl]->topology_key ||
            descs[i]->nodes.size() != descs[tmpl]->nodes.size())
          throw std::runtime_error("manifest groups " + paths[i] + " with a template of another topology (" +
                                   paths[tmpl] + ")");
        if (!resolved[i] || !resolved[tmpl]) return;
        diffs[i] = diff_against(*descs[tmpl], *descs[i]);
        diff_ready[i] = 1;
      });
    } catch (...) {
      std::lock_guard<std::mutex> lk(mu_);
      error_ = std::current_exception();
    }
    phase2_ms = ms_since(t0);
    std::lock_guard<std::mutex> lk(mu_);
    done_ = true;
    cv_.notify_all();
  });
}

void PendingLoads::wait() {
  std::unique_lock<std::mutex> lk(mu_);
  cv_.wait(lk, [this] { return done_; });
  if (error_) std::rethrow_exception(error_);
}

std::shared_ptr<RestoredGraph> PendingLoads::finish_one(size_t index) {
  if (index >= descs.size()) throw std::out_of_range("graph index out of range");
  wait();
  std::lock_guard<std::mutex> lk(finish_mu_);
  if (finished[index]) return results[index];
  // Graphs deferred by the background builds: resolve now (the engine has run
  // the warm-up that loads their kernels by the time it asks for them).
  const int gi = group_of[index];
  const int tmpl = group_template[gi];
  if (!resolved[tmpl]) {
    resolve_functions(*descs[tmpl]);
    resolved[tmpl] = 1;
  }
  if (!groups[gi]) {
    auto se = std::make_shared<SharedExec>();
    se->template_desc = descs[tmpl];
    se->built = build_graph(*descs[tmpl]);
    se->exec = instantiate(se->built->graph);
    groups[gi] = se;
  }
  if (!resolved[index]) {
    resolve_functions(*descs[index]);
    resolved[index] = 1;
  }
  if (static_cast<int>(index) != tmpl && !diff_ready[index]) {
    diffs[index] = diff_against(*descs[tmpl], *descs[index]);
    diff_ready[index] = 1;
  }
  // Allocator events are replayed in capture order: the cursor must walk the
  // same trajectory it walked on SAVE.
  const auto& ev = descs[index]->allocator_events_json;
  if (!ev.empty() && fb_events_replay_json(ev.data(), ev.size()) != FB_OK)
    throw std::runtime_error(std::string("replaying allocator events of ") + paths[index] + ": " +
                             fb_last_error());
  auto r = std::make_shared<RestoredGraph>();
  r->desc = descs[index];
  r->shared = groups[group_of[index]];
  r->path = paths[index];
  r->is_template = group_template[group_of[index]] == static_cast<int>(index);
  r->diff_nodes = diffs[index];
  r->ctx = ctx;
  if (r->is_template) {
    std::lock_guard<std::mutex> lk(r->shared->mu);
    if (!r->shared->current) r->shared->current = r.get();
  }
  results[index] = r;
  finished[index] = 1;
  return r;
}

PendingLoads::~PendingLoads() {
  if (worker_.joinable()) worker_.join();
}

}  // namespace fbc
