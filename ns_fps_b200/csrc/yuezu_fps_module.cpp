// yuezu_fps_module.cpp -- the drop-in Python surface of the engine.
//
// Same module contents as the reference binding
// (yuezu_fps/yuezu_fps_pybind.cpp:103-150): class SpaceRange with the same
// fields and methods, make_range, make_uniform_range, fps, fps_with_bbox and
// the five constants; the same argument names and defaults; the same return
// dtype (uint64 == size_t); the same error text for a wrong point shape.
// Everything computes through the C ABI of libnsfps.so (include/nsfps.h); the
// GIL is released around each sampling call.
//
// Deliberate differences (each turns a reference crash or misuse into a
// defined result):
//   * a non-contiguous float32 view is copied to a dense array first (the
//     reference reads the buffer as if it were dense);
//   * derived SpaceRange fields are recomputed from the current field values
//     on every use, so a default-constructed or edited SpaceRange and a dict
//     range work (the reference keeps the derived fields from construction
//     time and dereferences empty lookup tables for the other two);
//   * zero block counts raise RuntimeError (the reference divides by zero).
// Additions: `n_samples` is accepted as an alias of `sample_count` (the
// README's spelling), fps()/fps_with_bbox() take a `device` keyword, and
// fps_batched() samples many clouds in one call, optionally over many GPUs.
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <stdexcept>
#include <string>
#include <vector>

#include "nsfps.h"

namespace py = pybind11;

namespace {

using PointsArray = py::array_t<float, py::array::c_style | py::array::forcecast>;

struct SpaceRange {
  float min_x = 0, max_x = 0, min_y = 0, max_y = 0, min_z = 0, max_z = 0;
  uint32_t x_blocks = 0, y_blocks = 0, z_blocks = 0;

  nsfps_range c() const {
    return {min_x, max_x, min_y, max_y, min_z, max_z, x_blocks, y_blocks, z_blocks};
  }
  // src/yuezu_fps.cpp:7-11
  float block_size_x() const { return (max_x - min_x) / x_blocks; }
  float block_size_y() const { return (max_y - min_y) / y_blocks; }
  float block_size_z() const { return (max_z - min_z) / z_blocks; }
  // src/yuezu_fps.cpp:13-40
  static uint32_t bits_of(uint32_t b) {
    uint32_t bits = 0;
    while (bits < 32 && (1u << bits) < b) ++bits;
    return bits ? bits : 1;
  }
  uint32_t x_bits() const { return bits_of(x_blocks); }
  uint32_t y_bits() const { return bits_of(y_blocks); }
  uint32_t z_bits() const { return bits_of(z_blocks); }
  uint32_t total_bits() const { return x_bits() + y_bits() + z_bits(); }
  size_t total_blocks() const { return (size_t)x_blocks * y_blocks * z_blocks; }
};

[[noreturn]] void raise_last(int rc) {
  const std::string msg = nsfps_last_error();
  if (rc == NSFPS_ERR_ARG) throw std::runtime_error(msg);
  if (rc == NSFPS_ERR_OOM) throw std::runtime_error("out of memory: " + msg);
  throw std::runtime_error(msg);
}

PointsArray check_points(py::handle obj) {
  PointsArray a = PointsArray::ensure(obj);
  if (!a) throw std::runtime_error("Expected 2D array with shape (N, 3)");
  if (a.ndim() != 2 || a.shape(1) != 3)  // yuezu_fps_pybind.cpp:20-22
    throw std::runtime_error("Expected 2D array with shape (N, 3)");
  return a;
}

// parse_range (yuezu_fps_pybind.cpp:36-64): a SpaceRange or a dict with keys
// min_x..max_z and optional *_blocks (default 16).
SpaceRange parse_range(py::object obj) {
  if (py::isinstance<SpaceRange>(obj)) return obj.cast<SpaceRange>();
  if (py::isinstance<py::dict>(obj)) {
    py::dict d = obj.cast<py::dict>();
    SpaceRange r;
    try {
      r.min_x = d["min_x"].cast<float>();
      r.max_x = d["max_x"].cast<float>();
      r.min_y = d["min_y"].cast<float>();
      r.max_y = d["max_y"].cast<float>();
      r.min_z = d["min_z"].cast<float>();
      r.max_z = d["max_z"].cast<float>();
    } catch (const py::error_already_set &) {
      throw std::runtime_error(
          "range must be a SpaceRange object or a dict with keys: min_x, max_x, "
          "min_y, max_y, min_z, max_z");
    }
    r.x_blocks = d.contains("x_blocks") ? d["x_blocks"].cast<uint32_t>() : NSFPS_DEFAULT_X_BLOCKS;
    r.y_blocks = d.contains("y_blocks") ? d["y_blocks"].cast<uint32_t>() : NSFPS_DEFAULT_Y_BLOCKS;
    r.z_blocks = d.contains("z_blocks") ? d["z_blocks"].cast<uint32_t>() : NSFPS_DEFAULT_Z_BLOCKS;
    return r;
  }
  throw std::runtime_error(
      "range must be a SpaceRange object or a dict with keys: min_x, max_x, min_y, "
      "max_y, min_z, max_z");
}

py::array_t<uint64_t> to_array(const std::vector<uint64_t> &v, uint64_t len) {
  py::array_t<uint64_t> arr((py::ssize_t)len);
  if (len) std::memcpy(arr.mutable_data(), v.data(), sizeof(uint64_t) * len);
  return arr;
}

uint64_t resolve_k(py::object sample_count, py::object n_samples) {
  if (!sample_count.is_none() && !n_samples.is_none())
    throw py::type_error("pass either sample_count or n_samples, not both");
  py::object k = sample_count.is_none() ? n_samples : sample_count;
  if (k.is_none()) throw py::type_error("fps() missing required argument 'sample_count'");
  const long long v = k.cast<long long>();
  if (v < 0) throw py::type_error("sample_count must be non-negative");
  return (uint64_t)v;
}

py::array_t<uint64_t> fps(py::object points, py::object sample_count, py::object range,
                          py::object n_samples, int device) {
  PointsArray a = check_points(points);
  const uint64_t k = resolve_k(sample_count, n_samples);
  const uint64_t n = (uint64_t)a.shape(0);
  nsfps_range r{};
  const nsfps_range *rp = nullptr;
  if (!range.is_none()) {
    r = parse_range(range).c();
    rp = &r;
  }
  std::vector<uint64_t> out(std::max<uint64_t>(std::min(k, n), 1));
  uint64_t len = 0;
  int rc;
  {
    py::gil_scoped_release nogil;
    rc = nsfps_fps(a.data(), n, k, rp, out.data(), &len, device);
  }
  if (rc) raise_last(rc);
  return to_array(out, len);
}

py::array_t<uint64_t> fps_with_bbox(py::object points, py::object sample_count,
                                    uint32_t xb, uint32_t yb, uint32_t zb,
                                    py::object n_samples, int device) {
  PointsArray a = check_points(points);
  const uint64_t k = resolve_k(sample_count, n_samples);
  const uint64_t n = (uint64_t)a.shape(0);
  std::vector<uint64_t> out(std::max<uint64_t>(std::min(k, n), 1));
  uint64_t len = 0;
  int rc;
  {
    py::gil_scoped_release nogil;
    rc = nsfps_fps_with_bbox(a.data(), n, k, xb, yb, zb, out.data(), &len, device);
  }
  if (rc) raise_last(rc);
  return to_array(out, len);
}

py::list fps_batched(py::object clouds, uint64_t k, py::object range,
                     py::object devices) {
  std::vector<PointsArray> arrs;
  py::array maybe = py::array::ensure(clouds);
  if (maybe && maybe.ndim() == 3) {
    PointsArray a3 = PointsArray::ensure(clouds);
    if (!a3 || a3.shape(2) != 3) throw std::runtime_error("Expected array with shape (B, N, 3)");
    for (py::ssize_t b = 0; b < a3.shape(0); ++b)
      arrs.push_back(check_points(a3[py::int_(b)]));
  } else {
    for (py::handle h : clouds) arrs.push_back(check_points(h));
  }
  const uint64_t count = arrs.size();
  std::vector<const float *> ptrs(count);
  std::vector<uint64_t> ns(count), lens(count);
  std::vector<std::vector<uint64_t>> outs(count);
  std::vector<uint64_t *> optrs(count);
  for (uint64_t i = 0; i < count; ++i) {
    ptrs[i] = arrs[i].data();
    ns[i] = (uint64_t)arrs[i].shape(0);
    outs[i].resize(std::max<uint64_t>(std::min(k, ns[i]), 1));
    optrs[i] = outs[i].data();
  }
  std::vector<nsfps_range> rs;
  int per_cloud = 0;
  if (!range.is_none()) {
    if (py::isinstance<py::list>(range) || py::isinstance<py::tuple>(range)) {
      for (py::handle h : range) rs.push_back(parse_range(py::reinterpret_borrow<py::object>(h)).c());
      if (rs.size() != count) throw std::runtime_error("one range per cloud expected");
      per_cloud = 1;
    } else {
      rs.push_back(parse_range(range).c());
    }
  }
  std::vector<int> devs;
  if (devices.is_none()) devs.push_back(0);
  else for (py::handle h : devices) devs.push_back(h.cast<int>());
  if (devs.empty()) throw std::runtime_error("devices must not be empty");
  int rc;
  {
    py::gil_scoped_release nogil;
    rc = nsfps_fps_batched(ptrs.data(), ns.data(), count, k, rs.empty() ? nullptr : rs.data(),
                           per_cloud, optrs.data(), lens.data(), devs.data(), (int)devs.size());
  }
  if (rc) raise_last(rc);
  py::list res;
  for (uint64_t i = 0; i < count; ++i) res.append(to_array(outs[i], lens[i]));
  return res;
}

SpaceRange make_range(float min_x, float max_x, float min_y, float max_y, float min_z,
                      float max_z, uint32_t xb, uint32_t yb, uint32_t zb) {
  SpaceRange r;
  r.min_x = min_x; r.max_x = max_x;
  r.min_y = min_y; r.max_y = max_y;
  r.min_z = min_z; r.max_z = max_z;
  r.x_blocks = xb; r.y_blocks = yb; r.z_blocks = zb;
  return r;
}

}  // namespace

PYBIND11_MODULE(yuezu_fps_module, m) {
  m.doc() = "B200-native farthest point sampling with Morton-cell pruning "
            "(drop-in for yuezu_fps.yuezu_fps_module)";

  py::class_<SpaceRange>(m, "SpaceRange")
      .def(py::init<>())
      .def_readwrite("min_x", &SpaceRange::min_x)
      .def_readwrite("max_x", &SpaceRange::max_x)
      .def_readwrite("min_y", &SpaceRange::min_y)
      .def_readwrite("max_y", &SpaceRange::max_y)
      .def_readwrite("min_z", &SpaceRange::min_z)
      .def_readwrite("max_z", &SpaceRange::max_z)
      .def_readwrite("x_blocks", &SpaceRange::x_blocks)
      .def_readwrite("y_blocks", &SpaceRange::y_blocks)
      .def_readwrite("z_blocks", &SpaceRange::z_blocks)
      .def("block_size_x", &SpaceRange::block_size_x)
      .def("block_size_y", &SpaceRange::block_size_y)
      .def("block_size_z", &SpaceRange::block_size_z)
      .def("x_bits", &SpaceRange::x_bits)
      .def("y_bits", &SpaceRange::y_bits)
      .def("z_bits", &SpaceRange::z_bits)
      .def("total_bits", &SpaceRange::total_bits)
      .def("total_blocks", &SpaceRange::total_blocks)
      .def("__repr__", [](const SpaceRange &r) {
        return "SpaceRange(x=[" + std::to_string(r.min_x) + ", " + std::to_string(r.max_x) +
               "], y=[" + std::to_string(r.min_y) + ", " + std::to_string(r.max_y) +
               "], z=[" + std::to_string(r.min_z) + ", " + std::to_string(r.max_z) +
               "], blocks=" + std::to_string(r.x_blocks) + "x" + std::to_string(r.y_blocks) +
               "x" + std::to_string(r.z_blocks) + ")";
      });

  m.def("make_range", &make_range, py::arg("min_x"), py::arg("max_x"), py::arg("min_y"),
        py::arg("max_y"), py::arg("min_z"), py::arg("max_z"), py::arg("x_blocks"),
        py::arg("y_blocks"), py::arg("z_blocks"));

  m.def("make_uniform_range",
        [](float a, float b, float c, float d, float e, float f, uint32_t bpd) {
          return make_range(a, b, c, d, e, f, bpd, bpd, bpd);
        },
        py::arg("min_x"), py::arg("max_x"), py::arg("min_y"), py::arg("max_y"),
        py::arg("min_z"), py::arg("max_z"), py::arg("blocks_per_dim"));

  m.def("fps", &fps, py::arg("points"), py::arg("sample_count") = py::none(),
        py::arg("range") = py::none(), py::kw_only(), py::arg("n_samples") = py::none(),
        py::arg("device") = 0);

  m.def("fps_with_bbox", &fps_with_bbox, py::arg("points"),
        py::arg("sample_count") = py::none(), py::arg("x_blocks") = NSFPS_DEFAULT_X_BLOCKS,
        py::arg("y_blocks") = NSFPS_DEFAULT_Y_BLOCKS,
        py::arg("z_blocks") = NSFPS_DEFAULT_Z_BLOCKS, py::kw_only(),
        py::arg("n_samples") = py::none(), py::arg("device") = 0);

  m.def("fps_batched", &fps_batched, py::arg("clouds"), py::arg("sample_count"),
        py::arg("range") = py::none(), py::arg("devices") = py::none());

  m.def("device_count", []() {
    int c = 0;
    nsfps_device_count(&c);
    return c;
  });

  m.attr("DEFAULT_X_BLOCKS") = NSFPS_DEFAULT_X_BLOCKS;
  m.attr("DEFAULT_Y_BLOCKS") = NSFPS_DEFAULT_Y_BLOCKS;
  m.attr("DEFAULT_Z_BLOCKS") = NSFPS_DEFAULT_Z_BLOCKS;
  m.attr("MORTON_BLOCK_SIZE") = NSFPS_MORTON_BLOCK_SIZE;
  m.attr("CACHE_BLOCK_SIZE") = NSFPS_CACHE_BLOCK_SIZE;
}
