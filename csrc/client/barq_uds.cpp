// barq-uds: native command-line client for the Unix-domain-socket inference server.
//
// Parity: the reference's InferenceClient (advanced/src/uds_server.rs:300-395), a native client
// of the same server.  Wire format: every frame is a 4-byte big-endian length followed by a UTF-8
// JSON object.  A request {"id", "prompt", "max_tokens", "temperature"} is answered by a stream of
// {"id", "text", "tokens_generated", "ttft_ms", "total_time_ms", "done"} frames; the last one has
// done = true and, on failure, an "error" string.
//
//   barq-uds [--socket PATH] [--id ID] [--max-tokens N] [--temperature T] [--repeat R] [--json]
//            [--quiet] PROMPT
//   barq-uds --chat [--system TEXT] ...   interactive chat: one user turn per stdin line, the history
//            sent as OpenAI messages (rendered by the server's chat template); /exit ends it
//   barq-uds --health | --metrics         the engine's health frame (exit status 1 when unhealthy) or
//            its Prometheus metrics text
//
// The generated text streams to stdout as frames arrive (or, with --json, every frame's JSON one
// per line).  A summary line goes to stderr: tokens, TTFT and total time of each request, and for
// --repeat R > 1 the p50 / p99 of TTFT and the mean decode rate over the R requests, which are sent
// one after another on one connection.  Exit status: 0 on success, 1 when the server reported an
// error, 2 on a usage or connection error.
#include <sys/socket.h>
#include <sys/un.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <stdexcept>
#include <string>
#include <vector>

namespace {

constexpr uint32_t kMaxFrame = 16u << 20;

// ---------------------------------------------------------------- JSON (flat objects only)
// The server's frames are flat objects of strings, numbers, booleans and null.  Values of any
// other kind (arrays, nested objects) are skipped so that added fields do not break the client.
struct JsonValue {
  enum Kind { kNull, kBool, kNumber, kString, kOther } kind = kNull;
  bool b = false;
  double num = 0;
  std::string str;
};

class JsonReader {
 public:
  explicit JsonReader(const std::string& s) : s_(s) {}

  std::map<std::string, JsonValue> object() {
    std::map<std::string, JsonValue> out;
    ws();
    expect('{');
    ws();
    if (peek() == '}') {
      ++i_;
      return out;
    }
    for (;;) {
      ws();
      std::string key = string();
      ws();
      expect(':');
      ws();
      out[key] = value();
      ws();
      const char c = next();
      if (c == '}') break;
      if (c != ',') fail("expected , or }");
    }
    return out;
  }

 private:
  char peek() const { return i_ < s_.size() ? s_[i_] : '\0'; }
  char next() {
    if (i_ >= s_.size()) fail("unexpected end");
    return s_[i_++];
  }
  void expect(char c) {
    if (next() != c) fail(std::string("expected ") + c);
  }
  void ws() {
    while (i_ < s_.size() && (s_[i_] == ' ' || s_[i_] == '\t' || s_[i_] == '\n' || s_[i_] == '\r')) ++i_;
  }
  [[noreturn]] void fail(const std::string& what) const {
    throw std::runtime_error("bad JSON at byte " + std::to_string(i_) + ": " + what);
  }

  static void put_utf8(std::string& out, uint32_t cp) {
    if (cp < 0x80) {
      out += (char)cp;
    } else if (cp < 0x800) {
      out += (char)(0xC0 | (cp >> 6));
      out += (char)(0x80 | (cp & 0x3F));
    } else if (cp < 0x10000) {
      out += (char)(0xE0 | (cp >> 12));
      out += (char)(0x80 | ((cp >> 6) & 0x3F));
      out += (char)(0x80 | (cp & 0x3F));
    } else {
      out += (char)(0xF0 | (cp >> 18));
      out += (char)(0x80 | ((cp >> 12) & 0x3F));
      out += (char)(0x80 | ((cp >> 6) & 0x3F));
      out += (char)(0x80 | (cp & 0x3F));
    }
  }

  uint32_t hex4() {
    uint32_t v = 0;
    for (int k = 0; k < 4; ++k) {
      const char c = next();
      v <<= 4;
      if (c >= '0' && c <= '9') v |= c - '0';
      else if (c >= 'a' && c <= 'f') v |= c - 'a' + 10;
      else if (c >= 'A' && c <= 'F') v |= c - 'A' + 10;
      else fail("bad \\u escape");
    }
    return v;
  }

  std::string string() {
    expect('"');
    std::string out;
    for (;;) {
      const char c = next();
      if (c == '"') return out;
      if (c != '\\') {
        out += c;
        continue;
      }
      const char e = next();
      switch (e) {
        case '"': out += '"'; break;
        case '\\': out += '\\'; break;
        case '/': out += '/'; break;
        case 'b': out += '\b'; break;
        case 'f': out += '\f'; break;
        case 'n': out += '\n'; break;
        case 'r': out += '\r'; break;
        case 't': out += '\t'; break;
        case 'u': {
          uint32_t cp = hex4();
          if (cp >= 0xD800 && cp < 0xDC00) {  // high surrogate: a low one must follow
            if (next() != '\\' || next() != 'u') fail("unpaired surrogate");
            const uint32_t lo = hex4();
            if (lo < 0xDC00 || lo >= 0xE000) fail("unpaired surrogate");
            cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
          } else if (cp >= 0xDC00 && cp < 0xE000) {
            fail("unpaired surrogate");
          }
          put_utf8(out, cp);
          break;
        }
        default: fail("bad escape");
      }
    }
  }

  void skip_nested() {  // an array or object: skip to its matching close, honouring strings
    int depth = 0;
    do {
      const char c = peek();
      if (c == '"') {
        string();
        continue;
      }
      next();
      if (c == '[' || c == '{') ++depth;
      else if (c == ']' || c == '}') --depth;
    } while (depth > 0);
  }

  JsonValue value() {
    JsonValue v;
    const char c = peek();
    if (c == '"') {
      v.kind = JsonValue::kString;
      v.str = string();
    } else if (c == '{' || c == '[') {
      v.kind = JsonValue::kOther;
      skip_nested();
    } else if (s_.compare(i_, 4, "true") == 0) {
      v.kind = JsonValue::kBool, v.b = true, i_ += 4;
    } else if (s_.compare(i_, 5, "false") == 0) {
      v.kind = JsonValue::kBool, i_ += 5;
    } else if (s_.compare(i_, 4, "null") == 0) {
      i_ += 4;
    } else {
      const char* begin = s_.c_str() + i_;
      char* end = nullptr;
      v.num = std::strtod(begin, &end);
      if (end == begin) fail("bad value");
      v.kind = JsonValue::kNumber;
      i_ += (size_t)(end - begin);
    }
    return v;
  }

  const std::string& s_;
  size_t i_ = 0;
};

std::string json_quote(const std::string& s) {
  std::string out = "\"";
  for (unsigned char c : s) {
    switch (c) {
      case '"': out += "\\\""; break;
      case '\\': out += "\\\\"; break;
      case '\n': out += "\\n"; break;
      case '\r': out += "\\r"; break;
      case '\t': out += "\\t"; break;
      default:
        if (c < 0x20) {
          char buf[8];
          std::snprintf(buf, sizeof buf, "\\u%04x", c);
          out += buf;
        } else {
          out += (char)c;  // UTF-8 bytes pass through: JSON text is UTF-8
        }
    }
  }
  return out + "\"";
}

// ---------------------------------------------------------------- framing
bool write_all(int fd, const char* p, size_t n) {
  while (n > 0) {
    const ssize_t w = ::send(fd, p, n, MSG_NOSIGNAL);
    if (w < 0) {
      if (errno == EINTR) continue;
      return false;
    }
    p += w;
    n -= (size_t)w;
  }
  return true;
}

bool read_all(int fd, char* p, size_t n) {
  while (n > 0) {
    const ssize_t r = ::recv(fd, p, n, 0);
    if (r < 0 && errno == EINTR) continue;
    if (r <= 0) return false;
    p += r;
    n -= (size_t)r;
  }
  return true;
}

bool send_frame(int fd, const std::string& body) {
  const uint32_t n = (uint32_t)body.size();
  const char head[4] = {(char)(n >> 24), (char)(n >> 16), (char)(n >> 8), (char)n};
  return write_all(fd, head, 4) && write_all(fd, body.data(), body.size());
}

// false when the server closed the connection before a whole frame
bool recv_frame(int fd, std::string& body) {
  unsigned char head[4];
  if (!read_all(fd, (char*)head, 4)) return false;
  const uint32_t n = (uint32_t)head[0] << 24 | (uint32_t)head[1] << 16 | (uint32_t)head[2] << 8 | head[3];
  if (n > kMaxFrame) throw std::runtime_error("frame of " + std::to_string(n) + " bytes exceeds the 16 MiB limit");
  body.resize(n);
  return read_all(fd, &body[0], n);
}

// ---------------------------------------------------------------- client
struct Options {
  std::string socket_path = "/tmp/barq-inference.sock";
  std::string id = "req";
  std::string prompt;
  long max_tokens = 128;
  double temperature = 0.8;
  long repeat = 1;
  bool json = false, quiet = false, chat = false, health = false, metrics = false;
  std::string system;
};

struct Result {
  long tokens = 0;
  double ttft_ms = 0, total_ms = 0;
  std::string error;
};

// `input` is the request's prompt member: "\"prompt\":..." or "\"messages\":[...]" (JSON text).
Result run_request(int fd, const Options& o, const std::string& rid, const std::string& input,
                   std::string* reply = nullptr) {
  char num[64];
  std::string req = "{\"id\":" + json_quote(rid) + "," + input + ",\"max_tokens\":" + std::to_string(o.max_tokens) +
                    ",\"temperature\":";
  std::snprintf(num, sizeof num, "%.17g", o.temperature);
  req += num;
  req += "}";
  if (!send_frame(fd, req)) throw std::runtime_error("send failed: " + std::string(std::strerror(errno)));
  Result res;
  std::string body;
  for (;;) {
    if (!recv_frame(fd, body)) throw std::runtime_error("server closed the connection mid-stream");
    const auto fr = JsonReader(body).object();
    auto get = [&](const char* k) -> const JsonValue* {
      auto it = fr.find(k);
      return it == fr.end() ? nullptr : &it->second;
    };
    if (o.json) {
      std::fwrite(body.data(), 1, body.size(), stdout);
      std::fputc('\n', stdout);
    } else if (const JsonValue* t = get("text"); t && t->kind == JsonValue::kString && !o.quiet) {
      std::fwrite(t->str.data(), 1, t->str.size(), stdout);
    }
    if (const JsonValue* t = get("text"); reply && t && t->kind == JsonValue::kString) *reply += t->str;
    std::fflush(stdout);
    if (const JsonValue* v = get("tokens_generated"); v && v->kind == JsonValue::kNumber) res.tokens = (long)v->num;
    if (const JsonValue* v = get("ttft_ms"); v && v->kind == JsonValue::kNumber) res.ttft_ms = v->num;
    if (const JsonValue* v = get("total_time_ms"); v && v->kind == JsonValue::kNumber) res.total_ms = v->num;
    const JsonValue* done = get("done");
    if (done && done->kind == JsonValue::kBool && done->b) {
      if (const JsonValue* e = get("error"); e && e->kind == JsonValue::kString) res.error = e->str;
      return res;
    }
  }
}

// nearest-rank percentile of a non-empty sample
double percentile(std::vector<double> v, double p) {
  std::sort(v.begin(), v.end());
  const size_t rank = (size_t)std::ceil(p / 100.0 * (double)v.size());
  return v[std::min(v.size(), std::max<size_t>(rank, 1)) - 1];
}

[[noreturn]] void usage(const char* msg) {
  if (msg) std::fprintf(stderr, "barq-uds: %s\n", msg);
  std::fprintf(stderr,
               "usage: barq-uds [--socket PATH] [--id ID] [--max-tokens N] [--temperature T] [--repeat R]\n"
               "                [--json] [--quiet] PROMPT\n"
               "       barq-uds --chat [--system TEXT] [--socket PATH] [--max-tokens N] [--temperature T]\n"
               "                (one user turn per stdin line; the server renders the chat template)\n"
               "       barq-uds --health | --metrics [--socket PATH]   (the engine's health JSON / Prometheus text)\n");
  std::exit(2);
}

Options parse(int argc, char** argv) {
  Options o;
  bool have_prompt = false;
  for (int i = 1; i < argc; ++i) {
    const std::string a = argv[i];
    auto arg = [&]() -> std::string {
      if (i + 1 >= argc) usage(("missing value for " + a).c_str());
      return argv[++i];
    };
    auto num = [&](const std::string& s, bool integer) -> double {
      char* end = nullptr;
      const double v = integer ? (double)std::strtol(s.c_str(), &end, 10) : std::strtod(s.c_str(), &end);
      if (s.empty() || *end != '\0') usage(("bad number for " + a + ": " + s).c_str());
      return v;
    };
    if (a == "--socket") o.socket_path = arg();
    else if (a == "--id") o.id = arg();
    else if (a == "--max-tokens") o.max_tokens = (long)num(arg(), true);
    else if (a == "--temperature") o.temperature = num(arg(), false);
    else if (a == "--repeat") o.repeat = (long)num(arg(), true);
    else if (a == "--json") o.json = true;
    else if (a == "--quiet") o.quiet = true;
    else if (a == "--chat") o.chat = true;
    else if (a == "--health") o.health = true;
    else if (a == "--metrics") o.metrics = true;
    else if (a == "--system") o.system = arg();
    else if (a == "-h" || a == "--help") usage(nullptr);
    else if (!a.empty() && a[0] == '-' && a != "-") usage(("unknown option " + a).c_str());
    else if (have_prompt) usage("more than one prompt");
    else o.prompt = a, have_prompt = true;
  }
  if (!have_prompt && !o.chat && !o.health && !o.metrics) usage("no prompt");
  if (o.chat && (have_prompt || o.repeat != 1)) usage("--chat reads its turns from stdin (no PROMPT, no --repeat)");
  if (o.max_tokens < 0 || o.repeat < 1) usage("--max-tokens must be >= 0 and --repeat >= 1");
  return o;
}

}  // namespace

int main(int argc, char** argv) {
  const Options o = parse(argc, argv);
  sockaddr_un addr{};
  addr.sun_family = AF_UNIX;
  if (o.socket_path.size() >= sizeof(addr.sun_path)) usage("socket path too long");
  std::memcpy(addr.sun_path, o.socket_path.c_str(), o.socket_path.size() + 1);
  const int fd = ::socket(AF_UNIX, SOCK_STREAM, 0);
  if (fd < 0 || ::connect(fd, (const sockaddr*)&addr, sizeof addr) != 0) {
    std::fprintf(stderr, "barq-uds: cannot connect to %s: %s\n", o.socket_path.c_str(), std::strerror(errno));
    return 2;
  }
  if (o.health || o.metrics) {  // one query frame: the engine's health (JSON) or metrics (Prometheus text)
    const std::string what = o.health ? "health" : "metrics";
    std::string body;
    int status = 0;
    try {
      if (!send_frame(fd, "{\"id\":" + json_quote(what) + ",\"" + what + "\":true}") || !recv_frame(fd, body))
        throw std::runtime_error("no answer from the server");
      if (o.health) {
        std::fwrite(body.data(), 1, body.size(), stdout);
        std::fputc('\n', stdout);
        const auto fr = JsonReader(body).object();
        auto it = fr.find("healthy");
        if (it != fr.end() && it->second.kind == JsonValue::kBool && !it->second.b) status = 1;
      } else {
        const auto fr = JsonReader(body).object();
        auto it = fr.find("prometheus");
        if (it == fr.end() || it->second.kind != JsonValue::kString) throw std::runtime_error("no metrics in the answer");
        std::fwrite(it->second.str.data(), 1, it->second.str.size(), stdout);
      }
    } catch (const std::exception& e) {
      std::fprintf(stderr, "barq-uds: %s\n", e.what());
      status = 2;
    }
    ::close(fd);
    return status;
  }
  if (o.chat) {  // interactive multi-turn chat: the history travels as OpenAI messages
    std::vector<std::pair<std::string, std::string>> turns;
    if (!o.system.empty()) turns.emplace_back("system", o.system);
    int status = 0;
    char* line = nullptr;
    size_t cap = 0;
    ssize_t n;
    long turn = 0;
    try {
      while ((n = getline(&line, &cap, stdin)) >= 0) {
        std::string text(line, (size_t)n);
        while (!text.empty() && (text.back() == '\n' || text.back() == '\r')) text.pop_back();
        if (text == "/exit" || text == "/quit") break;
        if (text.empty()) continue;
        turns.emplace_back("user", text);
        std::string msgs = "\"messages\":[";
        for (size_t i = 0; i < turns.size(); ++i)
          msgs += (i ? ",{\"role\":" : "{\"role\":") + json_quote(turns[i].first) + ",\"content\":" +
                  json_quote(turns[i].second) + "}";
        msgs += "]";
        std::string reply;
        const Result res = run_request(fd, o, o.id + "-" + std::to_string(turn++), msgs, &reply);
        if (!o.json && !o.quiet) std::fputc('\n', stdout);
        std::fflush(stdout);
        if (!res.error.empty()) {
          std::fprintf(stderr, "barq-uds: error=%s\n", res.error.c_str());
          turns.pop_back();  // the failed turn is not part of the conversation
          status = 1;
          continue;
        }
        turns.emplace_back("assistant", reply);
      }
    } catch (const std::exception& e) {
      std::fprintf(stderr, "barq-uds: %s\n", e.what());
      status = 2;
    }
    std::free(line);
    ::close(fd);
    return status;
  }
  std::vector<double> ttft, rate;
  int status = 0;
  try {
    for (long r = 0; r < o.repeat; ++r) {
      const std::string rid = o.repeat == 1 ? o.id : o.id + "-" + std::to_string(r);
      const Result res = run_request(fd, o, rid, "\"prompt\":" + json_quote(o.prompt));
      if (!o.json && !o.quiet) std::fputc('\n', stdout);
      std::fprintf(stderr, "[%s] tokens=%ld ttft_ms=%.0f total_ms=%.0f%s%s\n", rid.c_str(), res.tokens, res.ttft_ms,
                   res.total_ms, res.error.empty() ? "" : " error=", res.error.c_str());
      if (!res.error.empty()) {
        status = 1;
        continue;
      }
      ttft.push_back(res.ttft_ms);
      if (res.tokens > 1 && res.total_ms > res.ttft_ms)
        rate.push_back((double)(res.tokens - 1) * 1e3 / (res.total_ms - res.ttft_ms));
    }
  } catch (const std::exception& e) {
    std::fprintf(stderr, "barq-uds: %s\n", e.what());
    ::close(fd);
    return 2;
  }
  ::close(fd);
  if (o.repeat > 1 && !ttft.empty()) {
    double mean_rate = 0;
    for (double x : rate) mean_rate += x;
    if (!rate.empty()) mean_rate /= (double)rate.size();
    std::fprintf(stderr, "summary: requests=%zu ttft_p50_ms=%.0f ttft_p99_ms=%.0f decode_tok_s=%.1f\n", ttft.size(),
                 percentile(ttft, 50), percentile(ttft, 99), mean_rate);
  }
  return status;
}
