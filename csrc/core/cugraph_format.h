// On-disk layout of the binary graph file (.cugraph, version 1).
//
// This layout is deliberately the same as the reference's
// (include/BinaryGraphFormat.h:14-229) so an archive directory has the same
// shape in both projects: a 64-byte header, a directory of 11 sections (24
// bytes each), then section payloads aligned to 8 bytes. Nodes are fixed
// 168-byte records (an 8-byte prefix plus a union sized by the memcpy variant).
// The structs below are our own declarations of that format; the
// static_asserts pin every size the format depends on.
#pragma once

#include <cstdint>

namespace fbc {
namespace bin {

constexpr char kMagic[8] = {'C', 'U', 'G', 'R', 'A', 'P', 'H', '\0'};
constexpr uint32_t kVersion = 1;

enum Section : uint32_t {
  S_STRINGS = 0,
  S_NODES = 1,
  S_DEPS = 2,
  S_PARAM_INDEX = 3,
  S_PARAM_DATA = 4,
  S_ARG_BUFFERS = 5,
  S_COMMON_ATTRS = 6,
  S_GENERATORS = 7,
  S_ALLOC_EVENTS = 8,
  S_OUTPUTS = 9,
  S_TOPOLOGY = 10,
  S_COUNT = 11,
};

enum HeaderFlag : uint32_t {
  HF_COMMON_ATTRS = 1u << 0,
  HF_DEPS = 1u << 1,
  HF_ALLOC_EVENTS = 1u << 2,
  HF_OUTPUTS = 1u << 3,
  HF_GENERATORS = 1u << 4,
  // Generator records carry the device addresses of the generator's graph
  // seed/offset words (GeneratorPtrRec) so a LOAD can relocate them; an
  // addition to v1, set only when a graph consumed random numbers.
  HF_GENERATOR_PTRS = 1u << 5,
  // Dependency records carry edge data (DepDataRec) because some edge is not
  // a plain full-completion dependency (programmatic dependent launch).
  HF_EDGE_DATA = 1u << 6,
};

#pragma pack(push, 1)
struct Header {
  char magic[8];
  uint32_t version;
  uint32_t flags;
  uint32_t num_nodes;
  uint32_t num_deps;
  uint32_t num_generators;
  uint32_t num_sections;
  uint32_t num_strings;
  uint8_t reserved[28];
};

struct SectionEntry {
  uint32_t type;
  uint32_t pad;
  uint64_t offset;
  uint64_t size;
};

struct KernelRec {
  uint32_t block[3];
  uint32_t grid[3];
  uint32_t smem;
  uint64_t binary_hash;
  uint32_t name_off;
  uint32_t name_len;
  int32_t max_dynamic_smem;
  int32_t preferred_carveout;
  int32_t cluster_sched_pref;
  int32_t required_cluster[3];
  uint32_t kna_flags;
  uint32_t cluster[3];
  uint32_t preferred_cluster[3];
  int32_t cluster_sched_policy;
  int32_t cooperative;
  int32_t priority;
  int32_t mem_sync_domain;
  uint8_t mem_sync_map_default;
  uint8_t mem_sync_map_remote;
  uint8_t attr_query_available;
  uint8_t pad;
  uint32_t preferred_smem_carveout;
  uint32_t param_index_off;  // byte offset into S_PARAM_INDEX
  uint32_t num_params;
  uint32_t arg_buffer_off;   // byte offset into S_ARG_BUFFERS, 0xFFFFFFFF if none
  uint32_t arg_buffer_size;
};

struct MemsetRec {
  uint64_t dst;
  uint32_t element_size;
  uint32_t pad0;
  uint64_t height;
  uint64_t pitch;
  uint32_t value;
  uint32_t pad1;
  uint64_t width;
};

struct MemcpyRec {
  uint64_t depth, height, width_bytes;
  uint64_t dst_device;
  uint64_t dst_height, dst_lod, dst_pitch, dst_x_bytes, dst_y, dst_z;
  int32_t dst_memory_type;
  int32_t pad0;
  uint64_t src_device;
  uint64_t src_height, src_lod, src_pitch, src_x_bytes, src_y, src_z;
  int32_t src_memory_type;
  int32_t pad1;
};

struct EventRec {
  int32_t event_id;
};

struct NodeRec {
  uint32_t node_id;
  uint8_t type;
  uint8_t pad[3];
  union {
    KernelRec kernel;
    MemsetRec memset;
    MemcpyRec memcpy;
    EventRec event;
  };
  uint8_t tail[168 - 8 - sizeof(MemcpyRec)];
};

struct ParamRec {
  uint32_t data_off;
  uint32_t size;
};

struct CommonAttrsRec {
  uint32_t flags;
  uint32_t cluster[3];
  uint32_t preferred_cluster[3];
  int32_t cluster_sched_policy;
  int32_t cooperative;
  int32_t priority;
  int32_t mem_sync_domain;
  uint8_t mem_sync_map_default;
  uint8_t mem_sync_map_remote;
  uint8_t attr_query_available;
  uint8_t pad;
  uint32_t preferred_smem_carveout;
};

struct DepDataRec {
  uint32_t from;
  uint32_t to;
  uint8_t from_port;
  uint8_t to_port;
  uint8_t type;
  uint8_t reserved;
};

struct GeneratorRec {
  uint64_t id;
  uint64_t seed;
  uint64_t wholegraph_increment;
};

struct GeneratorPtrRec {
  GeneratorRec base;
  uint64_t seed_ptr;
  uint64_t offset_ptr;
};

struct DepRec {
  uint32_t from;
  uint32_t to;
};
#pragma pack(pop)

static_assert(sizeof(Header) == 64, "header is 64 bytes");
static_assert(sizeof(SectionEntry) == 24, "section entry is 24 bytes");
static_assert(sizeof(KernelRec) == 136, "kernel record is 136 bytes");
static_assert(sizeof(MemsetRec) == 48, "memset record is 48 bytes");
static_assert(sizeof(MemcpyRec) == 152, "memcpy record is 152 bytes");
static_assert(sizeof(NodeRec) == 168, "node record is 168 bytes");
static_assert(sizeof(ParamRec) == 8, "param record is 8 bytes");
static_assert(sizeof(GeneratorRec) == 24, "generator record is 24 bytes");
static_assert(sizeof(GeneratorPtrRec) == 40, "generator record with pointers is 40 bytes");
static_assert(sizeof(DepRec) == 8, "dependency record is 8 bytes");
static_assert(sizeof(DepDataRec) == 12, "dependency record with edge data is 12 bytes");

}  // namespace bin
}  // namespace fbc
