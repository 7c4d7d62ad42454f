// The model descriptor, strix-stream/desc-v1: which placeable units exist (per layer: an expert slice or a layer
// blob), where their bytes live in the source files, and their xxh64. Format and validation rules follow the
// reference's desc.cpp so the same manifests load here.
#pragma once

#include <cstdint>
#include <string>
#include <vector>

#include "json.hpp"

namespace tsb {

enum class LayerKind { Dense, Moe, Blob };
enum class Tiers { Pinned, Disk, PinnedDisk, Pair };
enum class Order { Prefix, Ranked };

struct NamedBytes {
  std::string name;
  uint64_t bytes = 0;
};

struct Source {
  std::string name, path;
  uint64_t align = 4096;
};

// Unit u's piece: `bytes` at offset + u * stride of source `source`. A unit's bytes are its parts back to back.
struct Part {
  std::string name, format;
  int source = 0;
  uint64_t offset = 0, stride = 0, bytes = 0;
};

struct Router {
  std::string tensor, bias, format, score;
  uint32_t rows = 0, cols = 0;
};

struct Layer {
  int index = 0;
  LayerKind kind = LayerKind::Dense;
  uint64_t fixed_bytes = 0;
  int n_units = 0, top_k = 0, n_shared = 0;
  uint64_t unit_bytes = 0;
  std::vector<Part> parts;
  Router router;
  bool has_router = false;
  std::vector<uint64_t> hash;
  std::vector<double> benefit;
  bool streamable = true;
};

struct LookupTable {
  std::string name, placement;
  int source = 0;
  uint64_t offset = 0, rows = 0, row_bytes = 0;
};

struct Desc {
  std::string model, engine, routes;
  std::vector<NamedBytes> fixed_device, host_fixed;
  uint64_t state_bytes_per_position = 0, workspace_bytes_per_row = 0, unit_align = 256;
  std::vector<Source> sources;
  Order order = Order::Ranked;
  Tiers tiers = Tiers::PinnedDisk;
  uint32_t ring_slots = 0;
  std::vector<Layer> layers;
  std::vector<LookupTable> lookup_tables;
  // derived by desc_validate
  std::vector<int64_t> unit_base;
  int64_t total_units = 0;
  uint64_t max_unit_bytes = 0;
  int max_units_per_layer = 0;

  uint64_t unit_stride(int layer) const {
    const uint64_t b = layers[size_t(layer)].unit_bytes;
    return (b + unit_align - 1) / unit_align * unit_align;
  }
  uint64_t fixed_total() const;
};

Desc desc_from_json(const Json& j);
void desc_validate(Desc& d);
Json desc_to_json(const Desc& d);
const char* tiers_name(Tiers t);
const char* order_name(Order o);

}  // namespace tsb
