// The strix-stream/desc-v1 descriptor (desc.hpp): reading, checking and writing it. The format (keys, defaults,
// accepted values, limits, the rules a descriptor must satisfy) is the reference's (desc.cpp:126-441 there), so the
// same manifests load and write back the same document. Here every JSON object is read through a Scope that knows
// its path for messages and which keys it allows; each record type has a reader and a writer of its own.
#include "desc.hpp"

#include <algorithm>
#include <cstdio>
#include <functional>
#include <unordered_set>

#include "errors.hpp"

namespace tsb {
namespace {

const char* const kSchema = "strix-stream/desc-v1";
const char* const kSchemaRenamed = "tierstream/desc-v1";  // the same schema under the project's later name
constexpr uint64_t kLayerLimit = 4096, kUnitLimit = 1 << 16, kSourceLimit = 1024;
constexpr uint64_t kTotalLimit = uint64_t(1) << 56;

// One JSON object being read: its path (for messages) and its keys.
class Scope {
 public:
  Scope(const Json& j, std::string path) : j_(j), path_(std::move(path)) {}
  const std::string& path() const { return path_; }
  std::string at(const char* key) const { return path_ + "." + key; }
  // Keys outside `known` are refused, except adapter notes ("x-" prefixed).
  void known(std::initializer_list<const char*> keys) const {
    require(j_.is_object(), SS_E_DESC, path_ + ": expected an object");
    for (const auto& [k, v] : j_.obj) {
      (void)v;
      const bool note = k.compare(0, 2, "x-") == 0;
      require(note || std::any_of(keys.begin(), keys.end(), [&](const char* x) { return k == x; }), SS_E_DESC,
              path_ + ": unknown key \"" + k + "\"");
    }
  }
  const Json* opt(const char* key) const { return j_.find(key); }
  const Json& req(const char* key) const {
    const Json* v = j_.find(key);
    require(v != nullptr, SS_E_DESC, path_ + ": missing \"" + key + "\"");
    return *v;
  }
  uint64_t u64(const char* key) const { return json_u64(req(key), at(key)); }
  uint64_t u64(const char* key, uint64_t dflt) const {
    const Json* v = opt(key);
    return v ? json_u64(*v, at(key)) : dflt;
  }
  // An optional count with an upper limit.
  uint64_t count(const char* key, uint64_t dflt, uint64_t limit) const {
    const uint64_t v = u64(key, dflt);
    require(v <= limit, SS_E_DESC, at(key) + ": " + std::to_string(v) + " is above the limit " + std::to_string(limit));
    return v;
  }
  std::string str(const char* key) const { return json_str(req(key), at(key)); }
  std::string str(const char* key, const std::string& dflt) const {
    const Json* v = opt(key);
    return v ? json_str(*v, at(key)) : dflt;
  }
  // An optional array: f(element, its path) per element.
  void each(const char* key, const std::function<void(const Json&, const std::string&)>& f) const {
    const Json* v = opt(key);
    if (!v) return;
    require(v->is_array(), SS_E_DESC, at(key) + ": expected an array");
    for (size_t i = 0; i < v->arr.size(); ++i) f(v->arr[i], at(key) + "[" + std::to_string(i) + "]");
  }

 private:
  const Json& j_;
  std::string path_;
};

// Byte arithmetic of the checks: an overflow refuses the descriptor.
uint64_t sum_or_refuse(uint64_t a, uint64_t b, const std::string& where) {
  require(b <= UINT64_MAX - a, SS_E_DESC, where + ": byte arithmetic overflows 64 bits");
  return a + b;
}
uint64_t product_or_refuse(uint64_t a, uint64_t b, const std::string& where) {
  require(a == 0 || b <= UINT64_MAX / a, SS_E_DESC, where + ": byte arithmetic overflows 64 bits");
  return a * b;
}

bool is_pow2(uint64_t v) { return v && !(v & (v - 1)); }

// Tensor formats a part may name (and any "x-" adapter format).
bool format_known(const std::string& f) {
  static const std::unordered_set<std::string> names = {
      "F32",   "F16",   "BF16",  "FP8_E4M3", "FP8_E5M2", "EXL3",    "MXFP4",  "NVFP4",  "Q2_K",
      "Q3_K",  "Q4_K",  "Q5_K",  "Q6_K",     "Q8_0",     "Q4_0",    "Q4_1",   "Q5_0",   "Q5_1",
      "IQ1_S", "IQ1_M", "IQ2_XXS", "IQ2_XS", "IQ2_S",    "IQ3_XXS", "IQ3_S",  "IQ4_NL", "IQ4_XS",
      "TQ1_0", "TQ2_0", "I8",    "U8",    "mixed"};
  return names.count(f) > 0 || f.compare(0, 2, "x-") == 0;
}

// xxh64 values are 16 lowercase hex digits.
uint64_t parse_xxh(const std::string& s, const std::string& where) {
  require(s.size() == 16, SS_E_DESC, where + ": expected 16 hex digits");
  uint64_t v = 0;
  for (char c : s) {
    int nib = -1;
    if (c >= '0' && c <= '9') nib = c - '0';
    else if (c >= 'a' && c <= 'f') nib = 10 + (c - 'a');
    require(nib >= 0, SS_E_DESC, where + ": expected lowercase hex digits");
    v = v << 4 | uint64_t(nib);
  }
  return v;
}
std::string print_xxh(uint64_t v) {
  char buf[17];
  std::snprintf(buf, sizeof buf, "%016llx", static_cast<unsigned long long>(v));
  return buf;
}

const char* kind_name(LayerKind k) {
  return k == LayerKind::Dense ? "dense" : k == LayerKind::Moe ? "moe" : "blob";
}

// ---- readers ----
std::vector<NamedBytes> read_named(const Scope& s, const char* key) {
  std::vector<NamedBytes> out;
  s.each(key, [&](const Json& e, const std::string& path) {
    const Scope r(e, path);
    r.known({"name", "bytes"});
    out.push_back(NamedBytes{r.str("name"), r.u64("bytes")});
  });
  return out;
}

Part read_part(const Scope& r) {
  r.known({"name", "format", "source", "offset", "stride", "bytes"});
  Part p;
  p.name = r.str("name", "");
  p.format = r.str("format");
  p.source = int(r.count("source", 0, kSourceLimit));
  p.offset = r.u64("offset");
  p.bytes = r.u64("bytes");
  p.stride = r.u64("stride", p.bytes);
  return p;
}

Router read_router(const Scope& r) {
  r.known({"tensor", "bias", "format", "score", "rows", "cols"});
  Router x;
  x.tensor = r.str("tensor");
  x.bias = r.str("bias", "");
  x.format = r.str("format", "F32");
  x.score = r.str("score", "softmax");
  x.rows = uint32_t(r.count("rows", 0, kUnitLimit));
  x.cols = uint32_t(r.count("cols", 0, uint64_t(1) << 24));
  return x;
}

Layer read_layer(const Scope& r) {
  r.known({"index", "kind", "fixed_bytes", "n_units", "top_k", "n_shared", "unit_bytes", "parts", "router", "hash",
           "benefit", "streamable"});
  Layer l;
  const int64_t index = json_i64(r.req("index"), r.at("index"));
  require(index >= 0 && uint64_t(index) < kLayerLimit, SS_E_DESC, r.at("index") + ": 0..4095");
  l.index = int(index);
  const std::string kind = r.str("kind");
  if (kind == "dense") l.kind = LayerKind::Dense;
  else if (kind == "moe") l.kind = LayerKind::Moe;
  else if (kind == "blob") l.kind = LayerKind::Blob;
  else fail(SS_E_DESC, r.at("kind") + ": expected dense | moe | blob");
  l.fixed_bytes = r.u64("fixed_bytes", 0);
  l.n_units = int(r.count("n_units", l.kind == LayerKind::Blob ? 1 : 0, kUnitLimit));
  l.top_k = int(r.count("top_k", 0, kUnitLimit));
  l.n_shared = int(r.count("n_shared", 0, kUnitLimit));
  l.unit_bytes = r.u64("unit_bytes", 0);
  if (const Json* v = r.opt("streamable")) l.streamable = json_bool(*v, r.at("streamable"));
  r.each("parts", [&](const Json& e, const std::string& path) { l.parts.push_back(read_part(Scope(e, path))); });
  if (const Json* v = r.opt("router")) {
    l.router = read_router(Scope(*v, r.at("router")));
    l.has_router = true;
  }
  if (const Json* v = r.opt("hash"))
    require(v->is_array(), SS_E_DESC, r.at("hash") + ": expected an array of xxh64 hex strings");
  r.each("hash", [&](const Json& e, const std::string& path) { l.hash.push_back(parse_xxh(json_str(e, path), path)); });
  r.each("benefit", [&](const Json& e, const std::string& path) { l.benefit.push_back(json_f64(e, path)); });
  return l;
}

LookupTable read_table(const Scope& r) {
  r.known({"name", "source", "offset", "rows", "row_bytes", "placement"});
  LookupTable t;
  t.name = r.str("name");
  t.source = int(r.count("source", 0, kSourceLimit));
  t.offset = r.u64("offset", 0);
  t.rows = r.u64("rows");
  t.row_bytes = r.u64("row_bytes");
  t.placement = r.str("placement", "file");
  return t;
}

// ---- the rules a layer with units must satisfy; fills its unit bytes when omitted ----
void check_units(Layer& l, const std::string& path, const Desc& d) {
  require(!l.parts.empty(), SS_E_DESC, path + ".parts: a layer with units needs parts");
  uint64_t total = 0;
  for (size_t i = 0; i < l.parts.size(); ++i) {
    const Part& p = l.parts[i];
    const std::string pp = path + ".parts[" + std::to_string(i) + "]";
    require(p.bytes > 0, SS_E_DESC, pp + ".bytes: > 0");
    require(format_known(p.format), SS_E_DESC, pp + ".format: unknown format " + p.format);
    require(p.source >= 0 && size_t(p.source) < d.sources.size(), SS_E_DESC, pp + ".source: no such source");
    require(l.n_units == 1 || p.stride >= p.bytes, SS_E_DESC, pp + ".stride: >= bytes (units overlap)");
    total = sum_or_refuse(total, p.bytes, pp);
    // the last unit's piece ends inside 64-bit offsets
    const uint64_t last = sum_or_refuse(p.offset, product_or_refuse(uint64_t(l.n_units - 1), p.stride, pp), pp);
    (void)sum_or_refuse(last, p.bytes, pp);
  }
  if (!l.unit_bytes) l.unit_bytes = total;
  require(l.unit_bytes == total, SS_E_DESC,
          path + ".unit_bytes: " + std::to_string(l.unit_bytes) + " != sum of parts " + std::to_string(total));
  (void)product_or_refuse(sum_or_refuse(l.unit_bytes, d.unit_align, path), uint64_t(l.n_units), path);
  require(l.hash.empty() || l.hash.size() == size_t(l.n_units), SS_E_DESC, path + ".hash: one per unit");
  require(l.benefit.empty() || l.benefit.size() == size_t(l.n_units), SS_E_DESC, path + ".benefit: one per unit");
  require(!l.has_router || l.router.rows == 0 || l.router.rows == uint32_t(l.n_units), SS_E_DESC,
          path + ".router.rows: must equal n_units");
}

// ---- writers ----
Json named_json(const std::vector<NamedBytes>& v) {
  Json a = Json::array();
  for (const NamedBytes& n : v) {
    Json o = Json::object();
    o["name"] = Json::string(n.name);
    o["bytes"] = Json::number(n.bytes);
    a.push(o);
  }
  return a;
}

Json part_json(const Part& p) {
  Json o = Json::object();
  if (!p.name.empty()) o["name"] = Json::string(p.name);
  o["format"] = Json::string(p.format);
  o["source"] = Json::number(int64_t(p.source));
  for (const auto& [k, v] : {std::pair<const char*, uint64_t>{"offset", p.offset}, {"stride", p.stride},
                             {"bytes", p.bytes}})
    o[k] = Json::number(v);
  return o;
}

Json layer_json(const Layer& l) {
  Json o = Json::object();
  o["index"] = Json::number(int64_t(l.index));
  o["kind"] = Json::string(kind_name(l.kind));
  o["fixed_bytes"] = Json::number(l.fixed_bytes);
  if (l.n_units > 0) {  // a layer without units carries no unit fields
    o["n_units"] = Json::number(int64_t(l.n_units));
    o["unit_bytes"] = Json::number(l.unit_bytes);
    o["streamable"] = Json::boolean(l.streamable);
    Json parts = Json::array();
    for (const Part& p : l.parts) parts.push(part_json(p));
    o["parts"] = parts;
    if (!l.hash.empty()) {
      Json h = Json::array();
      for (uint64_t v : l.hash) h.push(Json::string(print_xxh(v)));
      o["hash"] = h;
    }
    if (!l.benefit.empty()) {
      Json b = Json::array();
      for (double v : l.benefit) b.push(Json::number(v));
      o["benefit"] = b;
    }
  }
  if (l.top_k) o["top_k"] = Json::number(int64_t(l.top_k));
  if (l.n_shared) o["n_shared"] = Json::number(int64_t(l.n_shared));
  if (l.has_router) {
    Json r = Json::object();
    const Router& x = l.router;
    for (const auto& [k, v] : {std::pair<const char*, const std::string*>{"tensor", &x.tensor}, {"bias", &x.bias},
                               {"format", &x.format}, {"score", &x.score}})
      if (k != std::string("bias") || !v->empty()) r[k] = Json::string(*v);  // an empty bias is left out
    r["rows"] = Json::number(uint64_t(x.rows));
    r["cols"] = Json::number(uint64_t(x.cols));
    o["router"] = r;
  }
  return o;
}

}  // namespace

const char* tiers_name(Tiers t) {
  static const char* const names[] = {"pinned", "disk", "pinned|disk", "pair"};  // in Tiers order
  const size_t i = size_t(t);
  return i < sizeof names / sizeof names[0] ? names[i] : "?";
}
const char* order_name(Order o) { return o == Order::Prefix ? "prefix" : "ranked"; }

uint64_t Desc::fixed_total() const {
  uint64_t t = 0;
  for (const NamedBytes& n : fixed_device) t += n.bytes;
  for (size_t L = 0; L < layers.size(); ++L)
    t += layers[L].fixed_bytes + (layers[L].streamable ? 0 : uint64_t(layers[L].n_units) * unit_stride(int(L)));
  return t;
}

Desc desc_from_json(const Json& j) {
  const Scope top(j, "desc");
  top.known({"schema", "model", "engine", "fixed_device", "host_fixed", "state_bytes_per_position",
             "workspace_bytes_per_row", "unit_align", "sources", "order", "tiers", "ring_slots", "routes", "layers",
             "lookup_tables"});
  const std::string schema = top.str("schema");
  require(schema == kSchema || schema == kSchemaRenamed, SS_E_DESC,
          std::string("desc.schema: expected \"") + kSchema + "\"");
  Desc d;
  d.model = top.str("model", "");
  d.engine = top.str("engine", "");
  d.fixed_device = read_named(top, "fixed_device");
  d.host_fixed = read_named(top, "host_fixed");
  d.state_bytes_per_position = top.u64("state_bytes_per_position", 0);
  d.workspace_bytes_per_row = top.u64("workspace_bytes_per_row", 0);
  d.unit_align = top.u64("unit_align", 256);
  d.ring_slots = uint32_t(top.count("ring_slots", 0, uint64_t(1) << 20));
  d.routes = top.str("routes", "");
  const std::string order = top.str("order", "ranked");
  require(order == "prefix" || order == "ranked", SS_E_DESC, "desc.order: expected prefix | ranked");
  d.order = order == "prefix" ? Order::Prefix : Order::Ranked;
  const std::string tiers = top.str("tiers", "pinned|disk");
  bool tiers_ok = false;
  for (Tiers t : {Tiers::Pinned, Tiers::Disk, Tiers::PinnedDisk, Tiers::Pair})
    if (tiers == tiers_name(t)) {
      d.tiers = t;
      tiers_ok = true;
    }
  require(tiers_ok, SS_E_DESC, "desc.tiers: expected pinned | disk | pinned|disk | pair");
  top.each("sources", [&](const Json& e, const std::string& path) {
    const Scope r(e, path);
    r.known({"name", "path", "align"});
    d.sources.push_back(Source{r.str("name", ""), r.str("path"), r.u64("align", 4096)});
  });
  const Json& layers = top.req("layers");
  require(layers.is_array(), SS_E_DESC, "desc.layers: expected an array");
  top.each("layers", [&](const Json& e, const std::string& path) { d.layers.push_back(read_layer(Scope(e, path))); });
  top.each("lookup_tables", [&](const Json& e, const std::string& path) {
    d.lookup_tables.push_back(read_table(Scope(e, path)));
  });
  desc_validate(d);
  return d;
}

void desc_validate(Desc& d) {
  require(!d.layers.empty() && d.layers.size() <= kLayerLimit, SS_E_DESC, "desc.layers: 1..4096 layers");
  require(is_pow2(d.unit_align), SS_E_DESC, "desc.unit_align: power of two");
  for (size_t s = 0; s < d.sources.size(); ++s)
    require(is_pow2(d.sources[s].align) && d.sources[s].align <= (uint64_t(1) << 20), SS_E_DESC,
            "desc.sources[" + std::to_string(s) + "].align: power of two <= 1 MiB");
  d.unit_base.assign(d.layers.size(), 0);
  d.total_units = 0;
  d.max_unit_bytes = 0;
  d.max_units_per_layer = 0;
  for (size_t i = 0; i < d.layers.size(); ++i) {
    Layer& l = d.layers[i];
    const std::string path = "desc.layers[" + std::to_string(i) + "]";
    require(l.index == int(i), SS_E_DESC, path + ".index: layers must be listed in order 0..n-1");
    switch (l.kind) {
      case LayerKind::Dense:
        require(l.n_units == 0 && l.parts.empty(), SS_E_DESC, path + ": a dense layer has no units (use fixed_bytes)");
        break;
      case LayerKind::Blob:
        require(l.n_units == 1, SS_E_DESC, path + ": a blob layer has exactly one unit");
        break;
      case LayerKind::Moe:
        require(l.n_units >= 1, SS_E_DESC, path + ": a moe layer needs n_units >= 1");
        require(l.top_k >= 1 && l.top_k <= l.n_units, SS_E_DESC, path + ".top_k: 1..n_units");
        break;
    }
    if (l.n_units > 0) {
      check_units(l, path, d);
      if (l.streamable) {
        d.max_unit_bytes = std::max(d.max_unit_bytes, l.unit_bytes);
        d.max_units_per_layer = std::max(d.max_units_per_layer, l.n_units);
      }
    }
    d.unit_base[i] = d.total_units;
    d.total_units += l.n_units;
  }
  // every byte the model names (with a page of slack per unit) stays below 64 PiB
  uint64_t device = 0, host = 0;
  for (const NamedBytes& n : d.fixed_device) device = sum_or_refuse(device, n.bytes, "desc.fixed_device");
  for (const NamedBytes& n : d.host_fixed) host = sum_or_refuse(host, n.bytes, "desc.host_fixed");
  uint64_t everything = sum_or_refuse(device, host, "desc");
  for (size_t L = 0; L < d.layers.size(); ++L) {
    const std::string path = "desc.layers[" + std::to_string(L) + "]";
    const uint64_t per = sum_or_refuse(d.layers[L].unit_bytes, 4096, path);
    everything = sum_or_refuse(everything, product_or_refuse(uint64_t(d.layers[L].n_units), per, path), path);
  }
  require(everything < kTotalLimit, SS_E_DESC, "desc: total bytes above 2^56 (64 PiB)");
  // the device's fixed bytes, non-streamable units included, stay within 64 bits
  for (size_t L = 0; L < d.layers.size(); ++L) {
    const std::string path = "desc.layers[" + std::to_string(L) + "]";
    device = sum_or_refuse(device, d.layers[L].fixed_bytes, path + ".fixed_bytes");
    if (!d.layers[L].streamable)
      device = sum_or_refuse(device, product_or_refuse(uint64_t(d.layers[L].n_units), d.unit_stride(int(L)), path),
                             path);
  }
  for (size_t i = 0; i < d.lookup_tables.size(); ++i) {
    const LookupTable& t = d.lookup_tables[i];
    const std::string path = "desc.lookup_tables[" + std::to_string(i) + "]";
    require(t.source >= 0 && size_t(t.source) < d.sources.size(), SS_E_DESC, path + ".source: no such source");
    require(t.placement == "file" || t.placement == "pinned" || t.placement == "device", SS_E_DESC,
            path + ".placement: file | pinned | device");
  }
}

Json desc_to_json(const Desc& d) {
  Json j = Json::object();
  j["schema"] = Json::string(kSchema);
  for (const auto& [k, v] : {std::pair<const char*, const std::string*>{"model", &d.model}, {"engine", &d.engine},
                             {"routes", &d.routes}})
    if (!v->empty()) j[k] = Json::string(*v);
  j["fixed_device"] = named_json(d.fixed_device);
  j["host_fixed"] = named_json(d.host_fixed);
  for (const auto& [k, v] : {std::pair<const char*, uint64_t>{"state_bytes_per_position", d.state_bytes_per_position},
                             {"workspace_bytes_per_row", d.workspace_bytes_per_row},
                             {"unit_align", d.unit_align},
                             {"ring_slots", d.ring_slots}})
    j[k] = Json::number(v);
  j["order"] = Json::string(order_name(d.order));
  j["tiers"] = Json::string(tiers_name(d.tiers));
  Json sources = Json::array();
  for (const Source& s : d.sources) {
    Json o = Json::object();
    if (!s.name.empty()) o["name"] = Json::string(s.name);
    o["path"] = Json::string(s.path);
    o["align"] = Json::number(s.align);
    sources.push(o);
  }
  j["sources"] = sources;
  Json layers = Json::array();
  for (const Layer& l : d.layers) layers.push(layer_json(l));
  j["layers"] = layers;
  Json tables = Json::array();
  for (const LookupTable& t : d.lookup_tables) {
    Json o = Json::object();
    o["name"] = Json::string(t.name);
    o["source"] = Json::number(int64_t(t.source));
    o["offset"] = Json::number(t.offset);
    o["rows"] = Json::number(t.rows);
    o["row_bytes"] = Json::number(t.row_bytes);
    o["placement"] = Json::string(t.placement);
    tables.push(o);
  }
  j["lookup_tables"] = tables;
  return j;
}

}  // namespace tsb
