// Restoring persisted graphs: topology groups share one instantiated
// template exec; other members of a group keep only the nodes whose launch
// parameters differ from the template and patch them into the exec with
// cuGraphExec*SetParams when they are launched.
//
// Parity: reference csrc/CUDAGraph.cpp:330-509 (on-demand replay),
// csrc/CUDAGraphParallel.cpp:1543-2099 (start_graph_builds / finish_*).
// Differences by design:
//  * switching members patches the *exec* directly with
//    cuGraphExecKernelNodeSetParams (only the differing nodes) and never calls
//    cudaDeviceSynchronize: exec updates only affect launches made after the
//    update, so work already queued on the GPU is unaffected;
//  * a member can be materialized into its own exec at any time (e.g. on a
//    background thread after the first token) to make later switches free;
//  * templates are built from the already-parsed binary data, never re-read.
#pragma once

#include <atomic>
#include <condition_variable>
#include <exception>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "graph_desc.h"

namespace fbc {

class RestoredGraph;

struct SharedExec {
  std::shared_ptr<GraphDesc> template_desc;
  std::unique_ptr<BuiltGraph> built;
  CUgraphExec exec = nullptr;
  std::mutex mu;
  const RestoredGraph* current = nullptr;  // member whose parameters are loaded
  uint64_t switches = 0;
  ~SharedExec();
};

class RestoredGraph {
 public:
  std::shared_ptr<GraphDesc> desc;
  std::shared_ptr<SharedExec> shared;
  std::vector<uint32_t> diff_nodes;  // positions that differ from the template
  std::string path;
  bool is_template = false;
  // Own exec after materialize(). Published with release ordering once fully
  // instantiated, so a launch on another thread either sees nothing (and
  // uses the shared exec) or the finished exec.
  std::unique_ptr<BuiltGraph> own_built;
  std::atomic<CUgraphExec> own_exec{nullptr};
  std::mutex materialize_mu;
  CUcontext ctx = nullptr;  // context of the restoring thread (made current by materialize)

  ~RestoredGraph();
  void launch(CUstream stream);
  void materialize();  // safe on any thread, concurrently with launch()
  size_t num_nodes() const { return desc ? desc->nodes.size() : 0; }
  uint64_t last_switch_ns = 0;
};

// Builds a stand-alone graph: resolve, build, instantiate (template of itself).
std::shared_ptr<RestoredGraph> restore_single(std::shared_ptr<GraphDesc> desc, const std::string& path);

// Compute the positions where member differs from tmpl (same topology).
std::vector<uint32_t> diff_against(const GraphDesc& tmpl, const GraphDesc& member);

class PendingLoads {
 public:
  std::vector<std::string> paths;
  std::vector<std::shared_ptr<GraphDesc>> descs;
  std::vector<int> group_of;
  std::vector<std::shared_ptr<SharedExec>> groups;
  std::vector<int> group_template;  // graph index of each group's template
  std::vector<std::vector<uint32_t>> diffs;
  std::vector<std::shared_ptr<RestoredGraph>> results;
  std::vector<char> finished;  // not vector<bool>: elements are written by finish_one
  // Kernels a graph names by entry only (images another library loads on
  // first use, e.g. cuBLAS kernels) may not be loaded yet when the background
  // builds run. Such graphs are resolved, and their group's template built,
  // when finish_one asks for them.
  std::vector<char> resolved;
  std::vector<char> diff_ready;
  std::vector<std::string> deferred_reason;
  double phase1_ms = 0, phase2_ms = 0;
  int num_threads = 4;
  CUcontext ctx = nullptr;

  void start_phase2();
  void wait();  // rethrows a phase-2 failure
  std::shared_ptr<RestoredGraph> finish_one(size_t index);
  ~PendingLoads();

 private:
  std::thread worker_;
  std::mutex mu_;
  std::condition_variable cv_;
  // Serialises finish_one: the finished check, the allocator-event replay and
  // the result store must happen once per graph and in one thread at a time.
  std::mutex finish_mu_;
  bool done_ = false;
  std::exception_ptr error_;
};

// rng_slot != 0: the generators' seed/offset words of every graph are moved to
// rng_slot / rng_slot + 8 (relocate_generator_words) as the graphs are read.
std::shared_ptr<PendingLoads> start_graph_builds(const std::vector<std::string>& paths, int num_threads,
                                                 uint64_t rng_slot = 0);

}  // namespace fbc
