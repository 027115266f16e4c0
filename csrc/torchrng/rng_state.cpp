// Read access to a CUDA generator's graph-capture state, for persisting
// graphs whose kernels draw random numbers.
//
// When torch captures a graph, kernels that use the Philox generator do not
// bake in the seed and offset: they read them from two device words owned by
// the generator's state (its "extragraph" seed and offset tensors), and every
// replay first writes the generator's seed and current offset there and then
// advances the offset by the graph's whole-graph increment. A persisted graph
// carries those two addresses and the increment; the restored graph's replay
// does the same three steps itself.
//
// The state hangs off at::CUDAGeneratorImpl::state_, a private member. Its
// fields are public (at::CUDAGeneratorState is a struct); the member pointer
// to state_ is obtained through an explicit template instantiation, which
// the language allows to name private members ([temp.spec.general]: access
// checking does not apply to the names in an explicit instantiation).
//
// Parity: the reference re-defines torch's generator registration functions
// to learn the same values (csrc/CUDAGraph.cpp:31-159); this module only
// reads them.
#include <ATen/cuda/CUDAGeneratorImpl.h>
#include <ATen/core/Generator.h>
#include <pybind11/pybind11.h>

namespace py = pybind11;

namespace {

struct StateMember {
  using type = c10::intrusive_ptr<at::CUDAGeneratorState> at::CUDAGeneratorImpl::*;
  friend type state_member(StateMember);
};

template <typename Tag, typename Tag::type Member>
struct ExposeMember {
  friend typename Tag::type state_member(Tag) { return Member; }
};

template struct ExposeMember<StateMember, &at::CUDAGeneratorImpl::state_>;

at::CUDAGeneratorState* default_state(int device) {
  const at::Generator& gen = at::cuda::detail::getDefaultCUDAGenerator(static_cast<c10::DeviceIndex>(device));
  auto* impl = at::check_generator<at::CUDAGeneratorImpl>(gen);
  return (impl->*state_member(StateMember{})).get();
}

uint64_t word_address(const at::TensorBase& t) {
  return t.defined() ? reinterpret_cast<uint64_t>(t.data_ptr()) : 0;
}

}  // namespace

PYBIND11_MODULE(_torchrng, m) {
  m.doc() = "Graph-capture state of torch's default CUDA generators (seed/offset words and increments).";
  m.def(
      "default_generator_graph_state",
      [](int device) {
        at::CUDAGeneratorState* s = default_state(device);
        py::dict d;
        d["seed"] = s->seed_;
        d["philox_offset"] = s->philox_offset_per_thread_;
        // After a capture ends this is the captured graph's whole-graph
        // increment (the capture prologue resets it, the epilogue reads it).
        d["offset_intragraph"] = s->offset_intragraph_;
        d["seed_ptr"] = word_address(s->seed_extragraph_);
        d["offset_ptr"] = word_address(s->offset_extragraph_);
        return d;
      },
      py::arg("device"));
}
