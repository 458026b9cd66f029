// Wire framing used by the worker pool and the raw-TCP gateway.
//
// Worker pipe protocol (openmini-server/src/service/worker/worker.rs:24-125,
// openmini-server/src/service/worker/pool.rs:191-320), kept byte-compatible:
//   command byte: 1 TASK, 2 SHUTDOWN, 3 HEARTBEAT, 4 LOAD_MODEL
//   TASK   frame: [1][u32 LE len][Task]        Task = [u64 LE id][u32 LE n][n bytes]
//   result frame: [u32 LE len][TaskResult]     TaskResult = [u64 LE id][u8 ok][u32 LE n][n bytes]
// Gateway request frame (openmini-server/src/service/server/gateway.rs:495-553):
//   [u32 BE len][type u8][session id 36 bytes][1 unused byte][stream u8][payload]
//   types: 1 chat, 2 image, 3 image-stream, 4 health
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <string>
#include <tuple>
#include <vector>

namespace py = pybind11;

namespace om_rt {

static void put_le32(std::string& b, uint32_t v) {
  for (int i = 0; i < 4; ++i) b.push_back((char)((v >> (8 * i)) & 0xFF));
}
static void put_le64(std::string& b, uint64_t v) {
  for (int i = 0; i < 8; ++i) b.push_back((char)((v >> (8 * i)) & 0xFF));
}
static uint32_t get_le32(const uint8_t* p) {
  return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}
static uint64_t get_le64(const uint8_t* p) {
  uint64_t v = 0;
  for (int i = 7; i >= 0; --i) v = (v << 8) | p[i];
  return v;
}

py::bytes encode_task(uint64_t id, const std::string& data) {
  std::string b;
  b.reserve(12 + data.size());
  put_le64(b, id);
  put_le32(b, (uint32_t)data.size());
  b += data;
  return py::bytes(b);
}

std::tuple<uint64_t, py::bytes> decode_task(const std::string& s) {
  const uint8_t* p = reinterpret_cast<const uint8_t*>(s.data());
  if (s.size() < 12) throw std::invalid_argument("Invalid task data: too short");
  const uint64_t id = get_le64(p);
  const uint32_t n = get_le32(p + 8);
  if (s.size() < 12 + (size_t)n) throw std::invalid_argument("Invalid task data: incomplete");
  return {id, py::bytes(s.substr(12, n))};
}

py::bytes encode_result(uint64_t id, bool ok, const std::string& data) {
  std::string b;
  put_le64(b, id);
  b.push_back(ok ? 1 : 0);
  put_le32(b, (uint32_t)data.size());
  b += data;
  return py::bytes(b);
}

std::tuple<uint64_t, bool, py::bytes> decode_result(const std::string& s) {
  const uint8_t* p = reinterpret_cast<const uint8_t*>(s.data());
  if (s.size() < 13) throw std::invalid_argument("Invalid result data: too short");
  const uint64_t id = get_le64(p);
  const bool ok = p[8] == 1;
  const uint32_t n = get_le32(p + 9);
  if (s.size() < 13 + (size_t)n) throw std::invalid_argument("Invalid result data: incomplete");
  return {id, ok, py::bytes(s.substr(13, n))};
}

// [cmd][u32 LE len][payload] for TASK / LOAD_MODEL, a bare [cmd] otherwise.
py::bytes encode_command(int cmd, const std::string& payload) {
  std::string b;
  b.push_back((char)cmd);
  if (cmd == 1 || cmd == 4) {
    put_le32(b, (uint32_t)payload.size());
    b += payload;
  }
  return py::bytes(b);
}

py::bytes encode_length_prefixed(const std::string& payload) {
  std::string b;
  put_le32(b, (uint32_t)payload.size());
  b += payload;
  return py::bytes(b);
}

// Incremental decoder for a stream of gateway frames.
class GatewayDecoder {
 public:
  explicit GatewayDecoder(uint32_t max_message) : max_(max_message) {}
  void feed(const std::string& data) { buf_ += data; }
  // Returns (type, session_id, stream, payload) or None when incomplete.
  py::object next() {
    if (buf_.size() < 4) return py::none();
    const uint8_t* p = reinterpret_cast<const uint8_t*>(buf_.data());
    const uint32_t len = ((uint32_t)p[0] << 24) | ((uint32_t)p[1] << 16) | ((uint32_t)p[2] << 8) | p[3];
    if (len > max_) {
      buf_.clear();
      throw std::invalid_argument("Message too large: " + std::to_string(len) + " bytes");
    }
    if (buf_.size() < 4 + (size_t)len) return py::none();
    std::string frame = buf_.substr(4, len);
    buf_.erase(0, 4 + (size_t)len);
    const int type = frame.empty() ? 0 : (uint8_t)frame[0];
    std::string session = frame.size() > 37 ? frame.substr(1, 36) : std::string();
    const bool stream = frame.size() > 38 && (uint8_t)frame[38] == 1;
    std::string payload = frame.size() > 39 ? frame.substr(39) : std::string();
    return py::make_tuple(type, session, stream, py::bytes(payload));
  }
  size_t buffered() const { return buf_.size(); }

 private:
  uint32_t max_;
  std::string buf_;
};

py::bytes encode_gateway(int type, const std::string& session, bool stream, const std::string& payload) {
  std::string f;
  f.push_back((char)type);
  std::string sid = session.substr(0, 36);
  sid.resize(36, ' ');
  f += sid;
  f.push_back(0);
  f.push_back(stream ? 1 : 0);
  f += payload;
  std::string b;
  const uint32_t n = (uint32_t)f.size();
  b.push_back((char)(n >> 24));
  b.push_back((char)(n >> 16));
  b.push_back((char)(n >> 8));
  b.push_back((char)n);
  b += f;
  return py::bytes(b);
}

}  // namespace om_rt

void bind_ipc(py::module_& m) {
  using namespace om_rt;
  m.attr("WORKER_CMD_TASK") = 1;
  m.attr("WORKER_CMD_SHUTDOWN") = 2;
  m.attr("WORKER_CMD_HEARTBEAT") = 3;
  m.attr("WORKER_CMD_LOAD_MODEL") = 4;
  m.def("encode_task", &encode_task);
  m.def("decode_task", &decode_task);
  m.def("encode_result", &encode_result);
  m.def("decode_result", &decode_result);
  m.def("encode_command", &encode_command, py::arg("cmd"), py::arg("payload") = std::string());
  m.def("encode_length_prefixed", &encode_length_prefixed);
  m.def("encode_gateway", &encode_gateway);
  py::class_<GatewayDecoder>(m, "GatewayDecoder")
      .def(py::init<uint32_t>(), py::arg("max_message") = 16u * 1024u * 1024u)
      .def("feed", &GatewayDecoder::feed)
      .def("next", &GatewayDecoder::next)
      .def("buffered", &GatewayDecoder::buffered);
}
