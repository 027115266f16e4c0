// Python bindings (module foundry_b200._C): region, event log, module
// registry, graph analysis/persistence/restore, and the kernel runtime that
// loads this repository's sm_100a cubins and launches them through the driver.
//
// Parity: reference csrc/binding.cpp:13-338 (module foundry.ops). The GIL is
// released around every call that may block on the driver or on the restore
// thread.
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <chrono>
#include <fstream>
#include <mutex>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

#include "../common/fb_driver.h"
#include "../common/fb_hook_api.h"
#include "graph_desc.h"
#include "restore.h"

namespace py = pybind11;
using namespace fbc;

namespace {

void check(fb_status s) {
  if (s != FB_OK) throw std::runtime_error(fb_last_error());
}

// ---- kernel runtime ----------------------------------------------------------

struct FuncInfo {
  std::vector<std::pair<size_t, size_t>> params;  // (offset, size)
  size_t total = 0;
};

std::mutex g_rt_mu;
std::unordered_map<CUfunction, FuncInfo> g_func_info;

const FuncInfo& func_info(CUfunction f) {
  std::lock_guard<std::mutex> lk(g_rt_mu);
  auto it = g_func_info.find(f);
  if (it != g_func_info.end()) return it->second;
  FuncInfo info;
  const FbDriver* d = fb_driver();
  for (size_t i = 0;; ++i) {
    size_t off = 0, sz = 0;
    CUresult rc = d->cuFuncGetParamInfo(f, i, &off, &sz);
    if (rc != CUDA_SUCCESS) break;
    info.params.emplace_back(off, sz);
    info.total = std::max(info.total, off + sz);
  }
  return g_func_info.emplace(f, std::move(info)).first->second;
}

// Packs Python arguments into the kernel's parameter layout: int -> little
// endian of the parameter's size, float -> float32 (4-byte slot) or float64,
// bytes -> copied verbatim (must match the size, e.g. a 128-byte CUtensorMap).
void pack_args(const FuncInfo& info, const py::sequence& args, std::vector<uint8_t>* buf,
               std::vector<void*>* ptrs) {
  if (static_cast<size_t>(py::len(args)) != info.params.size())
    throw std::runtime_error("kernel expects " + std::to_string(info.params.size()) + " arguments, got " +
                             std::to_string(py::len(args)));
  buf->assign(info.total + 16, 0);
  ptrs->clear();
  for (size_t i = 0; i < info.params.size(); ++i) {
    const size_t off = info.params[i].first, sz = info.params[i].second;
    uint8_t* dst = buf->data() + off;
    py::handle a = args[i];
    if (py::isinstance<py::bool_>(a)) {
      uint64_t v = a.cast<bool>() ? 1 : 0;
      memcpy(dst, &v, std::min<size_t>(sz, 8));
    } else if (py::isinstance<py::int_>(a)) {
      // Accept both signed and unsigned 64-bit values.
      uint64_t v;
      try {
        v = static_cast<uint64_t>(a.cast<int64_t>());
      } catch (const py::cast_error&) {
        v = a.cast<uint64_t>();
      }
      memcpy(dst, &v, std::min<size_t>(sz, 8));
    } else if (py::isinstance<py::float_>(a)) {
      double v = a.cast<double>();
      if (sz == 4) {
        float f = static_cast<float>(v);
        memcpy(dst, &f, 4);
      } else {
        memcpy(dst, &v, std::min<size_t>(sz, 8));
      }
    } else if (py::isinstance<py::bytes>(a)) {
      std::string s = a.cast<std::string>();
      if (s.size() != sz)
        throw std::runtime_error("argument " + std::to_string(i) + ": " + std::to_string(s.size()) +
                                 " bytes for a " + std::to_string(sz) + "-byte parameter");
      memcpy(dst, s.data(), sz);
    } else {
      throw std::runtime_error("argument " + std::to_string(i) + " has an unsupported type");
    }
  }
  for (const auto& p : info.params) ptrs->push_back(buf->data() + p.first);
}

py::tuple rt_load_image_file(const std::string& path) {
  std::ifstream f(path, std::ios::binary);
  if (!f) throw std::runtime_error("cannot open kernel image " + path);
  std::string bytes((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
  CUlibrary lib = nullptr;
  uint64_t hash = 0;
  {
    py::gil_scoped_release rel;
    check(fb_registry_load_image(bytes.data(), bytes.size(), path.c_str(), &lib, &hash));
  }
  return py::make_tuple(reinterpret_cast<uintptr_t>(lib), hash);
}

uintptr_t rt_get_function(uint64_t hash, const std::string& name, int max_dynamic_smem) {
  CUfunction f = nullptr;
  check(fb_registry_function(hash, name.c_str(), &f, nullptr));
  if (max_dynamic_smem > 0) {
    check_drv(fb_driver()->cuFuncSetAttribute(f, CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES,
                                               max_dynamic_smem),
              "cuFuncSetAttribute(max dynamic smem)");
  }
  return reinterpret_cast<uintptr_t>(f);
}

void rt_launch(uintptr_t fn, py::tuple grid, py::tuple block, unsigned smem, uintptr_t stream,
               py::sequence args, py::tuple cluster, bool pdl) {
  CUfunction f = reinterpret_cast<CUfunction>(fn);
  const FuncInfo& info = func_info(f);
  std::vector<uint8_t> buf;
  std::vector<void*> ptrs;
  pack_args(info, args, &buf, &ptrs);
  CUlaunchConfig cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.gridDimX = grid[0].cast<unsigned>();
  cfg.gridDimY = py::len(grid) > 1 ? grid[1].cast<unsigned>() : 1;
  cfg.gridDimZ = py::len(grid) > 2 ? grid[2].cast<unsigned>() : 1;
  cfg.blockDimX = block[0].cast<unsigned>();
  cfg.blockDimY = py::len(block) > 1 ? block[1].cast<unsigned>() : 1;
  cfg.blockDimZ = py::len(block) > 2 ? block[2].cast<unsigned>() : 1;
  cfg.sharedMemBytes = smem;
  cfg.hStream = reinterpret_cast<CUstream>(stream);
  CUlaunchAttribute attrs[2];
  memset(attrs, 0, sizeof(attrs));
  unsigned n = 0;
  if (py::len(cluster) > 0 && cluster[0].cast<unsigned>() > 1) {
    attrs[n].id = CU_LAUNCH_ATTRIBUTE_CLUSTER_DIMENSION;
    attrs[n].value.clusterDim.x = cluster[0].cast<unsigned>();
    attrs[n].value.clusterDim.y = py::len(cluster) > 1 ? cluster[1].cast<unsigned>() : 1;
    attrs[n].value.clusterDim.z = py::len(cluster) > 2 ? cluster[2].cast<unsigned>() : 1;
    ++n;
  }
  if (pdl) {
    // may start before the previous kernel of the stream completes; the
    // kernel waits for it with griddepcontrol.wait
    attrs[n].id = CU_LAUNCH_ATTRIBUTE_PROGRAMMATIC_STREAM_SERIALIZATION;
    attrs[n].value.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = n ? attrs : nullptr;
  cfg.numAttrs = n;
  check_drv(fb_driver()->cuLaunchKernelEx(&cfg, f, ptrs.data(), nullptr), "cuLaunchKernelEx");
}

py::bytes rt_make_tmap_2d(uint64_t ptr, int dtype, uint64_t inner, uint64_t outer, uint64_t row_stride_bytes,
                          uint32_t box_inner, uint32_t box_outer, int swizzle, int l2promo) {
  CUtensorMap m;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  check_drv(fb_driver()->cuTensorMapEncodeTiled(
                &m, static_cast<CUtensorMapDataType>(dtype), 2, reinterpret_cast<void*>(ptr), dims, strides,
                box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, static_cast<CUtensorMapSwizzle>(swizzle),
                static_cast<CUtensorMapL2promotion>(l2promo), CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE),
            "cuTensorMapEncodeTiled");
  return py::bytes(reinterpret_cast<const char*>(&m), sizeof(m));
}

py::bytes rt_make_tmap_3d(uint64_t ptr, int dtype, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t s1_bytes,
                          uint64_t s2_bytes, uint32_t b0, uint32_t b1, uint32_t b2, int swizzle) {
  CUtensorMap m;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {s1_bytes, s2_bytes};
  cuuint32_t box[3] = {b0, b1, b2};
  cuuint32_t estr[3] = {1, 1, 1};
  check_drv(fb_driver()->cuTensorMapEncodeTiled(
                &m, static_cast<CUtensorMapDataType>(dtype), 3, reinterpret_cast<void*>(ptr), dims, strides,
                box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, static_cast<CUtensorMapSwizzle>(swizzle),
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE),
            "cuTensorMapEncodeTiled");
  return py::bytes(reinterpret_cast<const char*>(&m), sizeof(m));
}

// Address of a __device__ global of an image (e.g. an error-status word).
py::tuple rt_get_global(uint64_t hash, const std::string& name) {
  CUlibrary lib = nullptr;
  check(fb_registry_library(hash, &lib));
  CUdeviceptr p = 0;
  size_t sz = 0;
  check_drv(fb_driver()->cuLibraryGetGlobal(&p, &sz, lib, name.c_str()), "cuLibraryGetGlobal");
  return py::make_tuple(static_cast<uint64_t>(p), sz);
}

int rt_func_attr(uintptr_t fn, int attr) {
  int v = 0;
  check_drv(fb_driver()->cuFuncGetAttribute(&v, static_cast<CUfunction_attribute>(attr),
                                            reinterpret_cast<CUfunction>(fn)),
            "cuFuncGetAttribute");
  return v;
}

// ---- raw VMM / multicast (symmetric memory substrate) --------------------------------

CUmemAllocationProp vmm_prop(int device, int handle_types) {
  CUmemAllocationProp prop;
  memset(&prop, 0, sizeof(prop));
  prop.type = CU_MEM_ALLOCATION_TYPE_PINNED;
  prop.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  prop.location.id = device;
  prop.requestedHandleTypes = static_cast<CUmemAllocationHandleType>(handle_types);
  return prop;
}

uint64_t vmm_granularity(int device) {
  CUmemAllocationProp prop = vmm_prop(device, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR);
  size_t g = 0;
  check_drv(fb_driver()->cuMemGetAllocationGranularity(&g, &prop, CU_MEM_ALLOC_GRANULARITY_RECOMMENDED),
            "cuMemGetAllocationGranularity");
  return g;
}

uint64_t vmm_create(uint64_t size, int device, int handle_types) {
  CUmemAllocationProp prop = vmm_prop(device, handle_types);
  CUmemGenericAllocationHandle h = 0;
  check_drv(fb_driver()->cuMemCreate(&h, size, &prop, 0), "cuMemCreate");
  return h;
}

int vmm_export_fd(uint64_t handle) {
  int fd = -1;
  check_drv(fb_driver()->cuMemExportToShareableHandle(&fd, handle, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0),
            "cuMemExportToShareableHandle");
  return fd;
}

uint64_t vmm_import_fd(int fd) {
  CUmemGenericAllocationHandle h = 0;
  check_drv(fb_driver()->cuMemImportFromShareableHandle(&h, reinterpret_cast<void*>(static_cast<intptr_t>(fd)),
                                                        CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR),
            "cuMemImportFromShareableHandle");
  return h;
}

uint64_t vmm_reserve(uint64_t base, uint64_t size, uint64_t align) {
  CUdeviceptr p = 0;
  check_drv(fb_driver()->cuMemAddressReserve(&p, size, align, static_cast<CUdeviceptr>(base), 0),
            "cuMemAddressReserve");
  if (base && p != base) {
    fb_driver()->cuMemAddressFree(p, size);
    throw std::runtime_error("could not reserve the symmetric span at the requested address (in use?)");
  }
  return p;
}

void vmm_map(uint64_t va, uint64_t size, uint64_t handle, uint64_t offset) {
  check_drv(fb_driver()->cuMemMap(static_cast<CUdeviceptr>(va), size, offset, handle, 0), "cuMemMap");
}

void vmm_set_access(uint64_t va, uint64_t size, std::vector<int> devices) {
  std::vector<CUmemAccessDesc> d(devices.size());
  for (size_t i = 0; i < devices.size(); ++i) {
    memset(&d[i], 0, sizeof(d[i]));
    d[i].location.type = CU_MEM_LOCATION_TYPE_DEVICE;
    d[i].location.id = devices[i];
    d[i].flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
  }
  check_drv(fb_driver()->cuMemSetAccess(static_cast<CUdeviceptr>(va), size, d.data(), d.size()), "cuMemSetAccess");
}

uint64_t mc_granularity(int num_devices, uint64_t size) {
  CUmulticastObjectProp p;
  memset(&p, 0, sizeof(p));
  p.numDevices = num_devices;
  p.size = size;
  p.handleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
  size_t g = 0;
  check_drv(fb_driver()->cuMulticastGetGranularity(&g, &p, CU_MULTICAST_GRANULARITY_RECOMMENDED),
            "cuMulticastGetGranularity");
  return g;
}

uint64_t mc_create(int num_devices, uint64_t size) {
  CUmulticastObjectProp p;
  memset(&p, 0, sizeof(p));
  p.numDevices = num_devices;
  p.size = size;
  p.handleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
  CUmemGenericAllocationHandle h = 0;
  check_drv(fb_driver()->cuMulticastCreate(&h, &p), "cuMulticastCreate");
  return h;
}

std::string events_json() {
  size_t n = fb_events_to_json(nullptr, 0);
  std::string s(n + 1, '\0');
  fb_events_to_json(&s[0], s.size());
  s.resize(n);
  return s;
}

}  // namespace

PYBIND11_MODULE(_C, m) {
  m.doc() = "foundry_b200 native core";

  // driver / hook status
  m.def("driver_path", []() { return std::string(fb_driver_path()); });
  m.def("driver_loaded", []() { return fb_driver()->loaded; });
  m.def("driver_is_mock", []() { return fb_driver()->is_mock; });
  m.def("hook_is_preloaded", []() { return fb_hook_is_preloaded() != 0; });
  m.def("intercepted_allocs", []() { return fb_hook_intercepted_allocs(); });
  m.def("last_error", []() { return std::string(fb_last_error()); });

  // region
  m.def("set_allocation_region", [](uint64_t base, uint64_t size) { check(fb_region_set(base, size)); },
        py::arg("base"), py::arg("size"));
  m.def("stop_allocation_region", []() { check(fb_region_stop()); });
  m.def("resume_allocation_region", []() { check(fb_region_resume()); });
  m.def("release_allocation_region", []() { check(fb_region_release()); });
  m.def("preallocate_region", [](uint64_t size) {
    fb_status s = fb_region_preallocate(size);
    if (s != FB_OK && s != FB_ERR_DRIVER) throw std::runtime_error(fb_last_error());
    return s == FB_OK;
  });
  m.def("free_preallocated_region", []() { check(fb_region_free_prealloc()); });
  m.def("get_current_alloc_offset", []() { return fb_region_get_offset(); });
  m.def("set_current_alloc_offset", [](uint64_t off) { check(fb_region_set_offset(off)); });
  m.def("region_base", []() { return fb_region_base(); });
  m.def("region_size", []() { return fb_region_size(); });
  m.def("region_active", []() { return fb_region_active() != 0; });
  m.def("region_granularity", []() { return fb_region_granularity(); });
  m.def("region_fallback_count", []() { return fb_region_fallback_count(); });
  m.def("region_alloc", [](uint64_t size) {
    uint64_t p = 0;
    check(fb_region_alloc(size, &p));
    return p;
  });
  m.def("region_free", [](uint64_t p) { check(fb_region_free(p)); });
  m.def("set_region_handle_types", [](int t) { fb_region_set_handle_types(t); });
  m.def("get_region_handle_types", []() { return fb_region_get_handle_types(); });
  m.def("set_region_peer_access", [](std::vector<int> devs) {
    fb_region_set_peer_access(devs.data(), static_cast<int>(devs.size()));
  });

  // events
  m.def("start_hook_record", []() { check(fb_events_start()); });
  m.def("end_hook_record", []() { check(fb_events_end()); });
  m.def("clear_hook_events", []() { fb_events_clear(); });
  m.def("hook_events_json", &events_json);
  m.def("replay_hook_events_json", [](const std::string& s) { check(fb_events_replay_json(s.data(), s.size())); });

  // registry
  m.def("pack_fatbins_to_folder", [](const std::string& folder) { check(fb_registry_pack(folder.c_str())); });
  m.def("load_cuda_modules_and_libraries", [](const std::string& folder) {
    py::gil_scoped_release rel;
    check(fb_registry_load_archive(folder.c_str()));
  });
  m.def("set_skip_fatbin_processing", [](bool e) { fb_registry_set_skip_processing(e ? 1 : 0); });
  m.def("set_pack_fatbins_on_exit", [](py::object folder) {
    if (folder.is_none()) fb_registry_set_pack_on_exit(nullptr);
    else fb_registry_set_pack_on_exit(folder.cast<std::string>().c_str());
  });
  m.def("registry_count", []() { return fb_registry_count(); });
  m.def("mark_binary_used", [](uint64_t h) { check(fb_registry_mark_used(h)); });
  m.def("init_nvshmem_modules", []() {
    char err[512] = {0};
    const int n = fb_registry_init_nvshmem(err, sizeof(err));
    if (n < 0) throw std::runtime_error(err);
    return n;
  });
  m.def("adopt_jit_function", [](uintptr_t fn, py::bytes image) {
    CUmodule mod = nullptr;
    check_drv(fb_driver()->cuFuncGetModule(&mod, reinterpret_cast<CUfunction>(fn)), "cuFuncGetModule");
    std::string b = image;
    uint64_t h = 0;
    check(fb_registry_adopt_module(mod, b.data(), b.size(), &h));
    return h;
  }, py::arg("function"), py::arg("image"));
  m.def("adopt_jit_module", [](uintptr_t mod, py::bytes image) {
    std::string b = image;
    uint64_t h = 0;
    check(fb_registry_adopt_module(reinterpret_cast<CUmodule>(mod), b.data(), b.size(), &h));
    return h;
  }, py::arg("module"), py::arg("image"));
  m.def("query_function_handle", [](uint64_t hash, const std::string& name) {
    CUfunction f = nullptr;
    check(fb_registry_function(hash, name.c_str(), &f, nullptr));
    return reinterpret_cast<uintptr_t>(f);
  });
  m.def("identify_function", [](uintptr_t fn) {
    uint64_t h = 0;
    char name[1024];
    check(fb_registry_identify(reinterpret_cast<CUfunction>(fn), &h, name, sizeof(name)));
    return py::make_tuple(h, std::string(name));
  });

  // kernel runtime
  m.def("load_image_file", &rt_load_image_file);
  m.def("get_function", &rt_get_function, py::arg("hash"), py::arg("name"), py::arg("max_dynamic_smem") = 0);
  m.def("launch", &rt_launch, py::arg("fn"), py::arg("grid"), py::arg("block"), py::arg("smem"),
        py::arg("stream"), py::arg("args"), py::arg("cluster") = py::tuple(), py::arg("pdl") = false);
  m.def("make_tmap_2d", &rt_make_tmap_2d, py::arg("ptr"), py::arg("dtype"), py::arg("inner"), py::arg("outer"),
        py::arg("row_stride_bytes"), py::arg("box_inner"), py::arg("box_outer"), py::arg("swizzle"),
        py::arg("l2promo") = 2);
  m.def("make_tmap_3d", &rt_make_tmap_3d);
  m.def("get_global", &rt_get_global);
  m.def("func_attr", &rt_func_attr);
  m.def("func_num_params", [](uintptr_t fn) { return func_info(reinterpret_cast<CUfunction>(fn)).params.size(); });

  // raw VMM + multicast (symmetric memory)
  m.def("vmm_granularity", &vmm_granularity);
  m.def("vmm_create", &vmm_create, py::arg("size"), py::arg("device"),
        py::arg("handle_types") = static_cast<int>(CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR));
  m.def("vmm_export_fd", &vmm_export_fd);
  m.def("vmm_import_fd", &vmm_import_fd);
  m.def("vmm_reserve", &vmm_reserve, py::arg("base"), py::arg("size"), py::arg("align") = 0);
  m.def("vmm_map", &vmm_map);
  m.def("vmm_set_access", &vmm_set_access);
  m.def("vmm_unmap", [](uint64_t va, uint64_t size) {
    check_drv(fb_driver()->cuMemUnmap(static_cast<CUdeviceptr>(va), size), "cuMemUnmap");
  });
  m.def("vmm_release", [](uint64_t h) { check_drv(fb_driver()->cuMemRelease(h), "cuMemRelease"); });
  m.def("vmm_free_va", [](uint64_t va, uint64_t size) {
    check_drv(fb_driver()->cuMemAddressFree(static_cast<CUdeviceptr>(va), size), "cuMemAddressFree");
  });
  m.def("mc_supported", []() { return fb_driver()->cuMulticastCreate != nullptr && !fb_driver()->is_mock; });
  m.def("mc_granularity", &mc_granularity);
  m.def("mc_create", &mc_create);
  m.def("mc_add_device", [](uint64_t mc, int device) {
    check_drv(fb_driver()->cuMulticastAddDevice(mc, device), "cuMulticastAddDevice");
  });
  m.def("mc_bind_mem", [](uint64_t mc, uint64_t mc_offset, uint64_t mem, uint64_t mem_offset, uint64_t size) {
    check_drv(fb_driver()->cuMulticastBindMem(mc, mc_offset, mem, mem_offset, size, 0), "cuMulticastBindMem");
  });
  m.def("mc_unbind", [](uint64_t mc, int device, uint64_t mc_offset, uint64_t size) {
    check_drv(fb_driver()->cuMulticastUnbind(mc, device, mc_offset, size), "cuMulticastUnbind");
  });
  m.def("device_attribute", [](int attr, int device) {
    int v = 0;
    check_drv(fb_driver()->cuDeviceGetAttribute(&v, static_cast<CUdevice_attribute>(attr), device),
              "cuDeviceGetAttribute");
    return v;
  });

  // graphs
  py::class_<GraphDesc, std::shared_ptr<GraphDesc>>(m, "GraphDesc")
      .def_property_readonly("num_nodes", [](const GraphDesc& g) { return g.nodes.size(); })
      .def_property_readonly("num_dependencies", [](const GraphDesc& g) { return g.deps.size(); })
      .def_property_readonly("topology_key", [](const GraphDesc& g) { return g.topology_key; })
      .def_property_readonly("num_events", [](const GraphDesc& g) { return g.num_events; })
      .def_property("allocator_events_json", [](const GraphDesc& g) { return g.allocator_events_json; },
                    [](GraphDesc& g, const std::string& s) { g.allocator_events_json = s; })
      .def_property("output_tensors_json", [](const GraphDesc& g) { return g.output_tensors_json; },
                    [](GraphDesc& g, const std::string& s) { g.output_tensors_json = s; })
      .def("kernel_names", [](const GraphDesc& g) {
        std::vector<std::string> v;
        for (const auto& n : g.nodes)
          if (n.type == NodeType::Kernel) v.push_back(n.kernel.func_name);
        return v;
      })
      .def("edges", [](const GraphDesc& g) {
        // (from, to, from_port, to_port, type) per dependency; ports and type 0 = a plain edge
        py::list out;
        for (size_t i = 0; i < g.deps.size(); ++i) {
          const bool has = !g.edge_data.empty();
          out.append(py::make_tuple(g.deps[i].first, g.deps[i].second, has ? g.edge_data[i].from_port : 0,
                                    has ? g.edge_data[i].to_port : 0, has ? g.edge_data[i].type : 0));
        }
        return out;
      })
      .def("node_types", [](const GraphDesc& g) {
        std::vector<std::string> v;
        for (const auto& n : g.nodes) v.push_back(node_type_name(n.type));
        return v;
      })
      .def("kernel_params", [](const GraphDesc& g, size_t i) {
        const Node& n = g.nodes.at(i);
        py::list out;
        for (const auto& p : n.kernel.params) out.append(py::bytes(reinterpret_cast<const char*>(p.data()), p.size()));
        return out;
      })
      .def_property(
          "generators",
          [](const GraphDesc& g) {
            py::list out;
            for (const auto& gen : g.generators) {
              py::dict d;
              d["id"] = gen.id;
              d["seed"] = gen.seed;
              d["wholegraph_increment"] = gen.wholegraph_increment;
              d["seed_ptr"] = gen.seed_ptr;
              d["offset_ptr"] = gen.offset_ptr;
              out.append(d);
            }
            return out;
          },
          [](GraphDesc& g, const py::list& gens) {
            std::vector<Generator> v;
            for (const auto& item : gens) {
              const py::dict d = item.cast<py::dict>();
              Generator gen;
              gen.id = d.contains("id") ? d["id"].cast<uint64_t>() : 0;
              gen.seed = d["seed"].cast<uint64_t>();
              gen.wholegraph_increment = d["wholegraph_increment"].cast<uint64_t>();
              gen.seed_ptr = d.contains("seed_ptr") ? d["seed_ptr"].cast<uint64_t>() : 0;
              gen.offset_ptr = d.contains("offset_ptr") ? d["offset_ptr"].cast<uint64_t>() : 0;
              v.push_back(gen);
            }
            g.generators = std::move(v);
          })
      .def("relocate_generator_words", [](GraphDesc& g, uint64_t slot) { return relocate_generator_words(g, slot); })
      .def("to_json", [](const GraphDesc& g) { return to_json(g).dump(); })
      .def("save", [](GraphDesc& g, const std::string& json_path) {
        py::gil_scoped_release rel;
        std::string text = to_json(g).dump();
        {
          std::ofstream f(json_path, std::ios::trunc);
          if (!f) throw std::runtime_error("cannot write " + json_path);
          f << text;
        }
        write_binary(g, cugraph_path_for(json_path));
      });
  m.def("analyze_graph", [](uintptr_t graph) {
    py::gil_scoped_release rel;
    return analyze_graph(reinterpret_cast<CUgraph>(graph));
  });
  m.def("read_graph_file", [](const std::string& path) {
    py::gil_scoped_release rel;
    return read_graph_file(path);
  });
  m.def("read_binary_graph", [](const std::string& path) { return read_binary(path); });
  m.def("graph_from_json_text", [](const std::string& text) { return from_json(fb::json::parse(text)); });
  m.def("diff_against", [](const GraphDesc& a, const GraphDesc& b) { return diff_against(a, b); });
  // Builds a live (non-instantiated) CUgraph from a description: used to create
  // synthetic graphs for tests and tools. The caller owns the returned handle.
  m.def("build_live_graph", [](std::shared_ptr<GraphDesc> d) {
    resolve_functions(*d);
    auto b = build_graph(*d);
    CUgraph g = b->graph;
    b->graph = nullptr;
    b->events.clear();  // owned by the graph's event nodes for the test's lifetime
    return reinterpret_cast<uintptr_t>(g);
  });
  m.def("destroy_graph", [](uintptr_t g) {
    if (g) fb_driver()->cuGraphDestroy(reinterpret_cast<CUgraph>(g));
  });
  m.def("recompute_topology_key", [](GraphDesc& g) {
    g.topology_key = compute_topology_key(g);
    return g.topology_key;
  });

  py::class_<RestoredGraph, std::shared_ptr<RestoredGraph>>(m, "RestoredGraph")
      .def("launch", [](RestoredGraph& g, uintptr_t stream) {
        py::gil_scoped_release rel;
        g.launch(reinterpret_cast<CUstream>(stream));
      })
      .def("materialize", [](RestoredGraph& g) {
        py::gil_scoped_release rel;
        g.materialize();
      })
      .def_property_readonly("desc", [](const RestoredGraph& g) { return g.desc; })
      .def_property_readonly("path", [](const RestoredGraph& g) { return g.path; })
      .def_property_readonly("is_template", [](const RestoredGraph& g) { return g.is_template; })
      .def_property_readonly("num_diff_nodes", [](const RestoredGraph& g) { return g.diff_nodes.size(); })
      .def_property_readonly("materialized", [](const RestoredGraph& g) { return g.own_exec.load() != nullptr; })
      .def_property_readonly("last_switch_ns", [](const RestoredGraph& g) { return g.last_switch_ns; })
      .def_property_readonly("exec_handle", [](const RestoredGraph& g) {
        CUgraphExec e = g.own_exec.load();
        return reinterpret_cast<uintptr_t>(e ? e : (g.shared ? g.shared->exec : nullptr));
      })
      .def_property_readonly("output_tensors_json", [](const RestoredGraph& g) { return g.desc->output_tensors_json; });
  m.def("load_graph", [](const std::string& path, uint64_t rng_slot) {
    py::gil_scoped_release rel;
    auto desc = read_graph_file(path);
    if (rng_slot) relocate_generator_words(*desc, rng_slot);
    const auto& ev = desc->allocator_events_json;
    if (!ev.empty() && fb_events_replay_json(ev.data(), ev.size()) != FB_OK)
      throw std::runtime_error(fb_last_error());
    return restore_single(desc, path);
  }, py::arg("path"), py::arg("rng_slot") = 0);

  py::class_<PendingLoads, std::shared_ptr<PendingLoads>>(m, "PendingGraphLoads")
      .def_property_readonly("num_graphs", [](const PendingLoads& p) { return p.paths.size(); })
      .def_property_readonly("num_groups", [](const PendingLoads& p) { return p.group_template.size(); })
      .def_property_readonly("phase1_ms", [](const PendingLoads& p) { return p.phase1_ms; })
      .def_property_readonly("phase2_ms", [](const PendingLoads& p) { return p.phase2_ms; })
      .def("wait", [](PendingLoads& p) {
        py::gil_scoped_release rel;
        p.wait();
      })
      .def("finish_one", [](PendingLoads& p, size_t i) {
        py::gil_scoped_release rel;
        return p.finish_one(i);
      });
  m.def("start_graph_builds", [](const std::vector<std::string>& paths, int num_threads, uint64_t rng_slot) {
    py::gil_scoped_release rel;
    return start_graph_builds(paths, num_threads, rng_slot);
  }, py::arg("paths"), py::arg("num_threads") = 4, py::arg("rng_slot") = 0);
}
