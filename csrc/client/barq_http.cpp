// barq-http: native OpenAI-compatible HTTP front end for the barq engine.
//
// Parity: the reference's front end serves the OpenAI routes from its CLI binary
// (cli/src/server.rs:297-370: GET /, GET /v1/models, POST /v1/completions, /v1/chat/completions,
// /v1/responses, OPTIONS for CORS, per-IP rate limiting with 429, SSE streaming) and talks to the
// inference side over a local socket (advanced/src/uds_server.rs).  This binary is that front end
// in C++: it owns the HTTP side (parsing, keep-alive, CORS, rate limiting, SSE framing, stop
// strings, request ids, Prometheus counters) and forwards every generation to the engine's UDS
// server (`barq server --socket PATH`), one socket connection per request.  Tokenization, chat
// templates and sampling stay in the engine process.
//
//   barq-http --socket PATH [--socket PATH ...] [--host 0.0.0.0] [--port 8080] [--model-id NAME] [--rpm N]
//             [--max-conns N] [--engine-timeout S] [--drain-timeout S] [--api-key KEY] [--quiet]
//
// With --api-key (or BARQ_API_KEY in the environment) the /v1 routes answer 401 unless the request
// carries "Authorization: Bearer KEY"; /, /health and /metrics stay open.
//
// With several --socket engines (e.g. one engine process per GPU) each request goes to the engine
// with the fewest requests in flight that accepts the connection (one that refuses is skipped for
// 5 s, and the request fails over); /health lists every engine and /metrics labels their samples.
//
// SIGTERM / SIGINT stop it gracefully: the listening socket closes and generations in flight get up
// to --drain-timeout seconds (default 30) to finish before the process exits.
//
// Routes:
//   GET  /                       server info
//   GET  /v1/models              the served model id
//   GET  /health                 the engine's health frame: 200 ok, 503 degraded or unreachable
//   GET  /metrics                Prometheus text: this front end's counters, then the engine's
//   POST /v1/completions         prompt (string or token ids)
//   POST /v1/chat/completions    messages (rendered by the engine's chat template)
//   POST /v1/responses           input (string or messages) / prompt / messages, max_output_tokens
//   POST /v1/embeddings          input (string, strings, token ids or lists of them)
//   POST /tokenize, /detokenize  {"content"[, "add_special"]} -> {"tokens"}; {"tokens"} -> {"content"}
//   OPTIONS *                    204 with CORS headers
// Request fields forwarded to the engine: max_tokens, temperature, top_k, top_p, min_p, seed,
// repetition / frequency / presence penalties, response_format, grammar, tools / tool_choice (the
// engine renders the tool prompt and reports a recognized call, returned here as tool_calls).
// logprobs / top_logprobs are forwarded too and the engine's per-token entries come back as the
// OpenAI chat or completions logprob objects.  Handled here: stream, stream_options.include_usage,
// stop (string or list; text is held back while it could still be the start of a stop string, so
// no stop text is ever sent), n (1..16, not with stream).
// Errors: 400 invalid request, 404 unknown route, 405 wrong method, 413 / 431 oversized, 429 rate
// limited, 502 engine unreachable, 503 engine queue full or connection limit, 500 engine failure;
// the body is {"error": {"message", "type"}} as in the Python server.
#include <arpa/inet.h>
#include <netinet/in.h>
#include <netinet/tcp.h>
#include <poll.h>
#include <signal.h>
#include <sys/socket.h>
#include <sys/time.h>
#include <sys/un.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cctype>
#include <cerrno>
#include <cmath>
#include <chrono>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <ctime>
#include <functional>
#include <map>
#include <mutex>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

#include "json_lite.h"

namespace {

using barqjson::Value;

constexpr size_t kMaxHeaderBytes = 32 << 10;
constexpr size_t kMaxBodyBytes = 8 << 20;
constexpr uint32_t kMaxFrame = 16u << 20;

struct Options {
  std::string host = "0.0.0.0";
  int port = 8080;
  std::vector<std::string> sockets;  // engine UDS servers (one per engine process; requests are balanced)
  std::string model_id = "barq";
  int rpm = 0;          // requests per minute per client address (0: no limit)
  int max_conns = 256;  // concurrent connections
  int engine_timeout_s = 600;
  int drain_s = 30;  // on SIGTERM / SIGINT: stop accepting, let requests in flight finish this long
  std::string api_key;  // non-empty: /v1 routes need "Authorization: Bearer <key>"
  bool quiet = false;
};
volatile sig_atomic_t g_stop = 0;
void on_stop_signal(int) { g_stop = 1; }
Options g_opt;

double now_s() {
  return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

// ---------------------------------------------------------------- counters (Prometheus text)
struct Counters {
  std::atomic<uint64_t> requests{0}, ok{0}, client_errors{0}, server_errors{0}, rate_limited{0};
  std::atomic<uint64_t> prompt_tokens{0}, completion_tokens{0};
  std::atomic<uint64_t> ttft_us{0}, ttft_n{0}, latency_us{0}, latency_n{0};
  std::atomic<int64_t> active{0}, peak_active{0}, connections{0};

  void begin() {
    const int64_t a = ++active;
    int64_t p = peak_active.load();
    while (a > p && !peak_active.compare_exchange_weak(p, a)) {
    }
  }
  std::string prometheus() const {
    std::string s;
    auto line = [&](const char* name, const char* type, const char* help, double v) {
      char buf[64];
      std::snprintf(buf, sizeof buf, "%.17g", v);
      s += std::string("# HELP ") + name + " " + help + "\n# TYPE " + name + " " + type + "\n" + name + " " + buf + "\n";
    };
    line("barq_http_requests_total", "counter", "Generation requests received.", (double)requests);
    line("barq_http_requests_ok_total", "counter", "Generation requests answered with 200.", (double)ok);
    line("barq_http_client_errors_total", "counter", "Requests answered with a 4xx status.", (double)client_errors);
    line("barq_http_server_errors_total", "counter", "Requests answered with a 5xx status.", (double)server_errors);
    line("barq_http_rate_limited_total", "counter", "Requests refused by the rate limiter.", (double)rate_limited);
    line("barq_http_prompt_tokens_total", "counter", "Prompt tokens of completed requests.", (double)prompt_tokens);
    line("barq_http_completion_tokens_total", "counter", "Generated tokens of completed requests.",
         (double)completion_tokens);
    line("barq_http_ttft_seconds_sum", "counter", "Sum of time to first token.", (double)ttft_us * 1e-6);
    line("barq_http_ttft_seconds_count", "counter", "Requests with a first token.", (double)ttft_n);
    line("barq_http_request_seconds_sum", "counter", "Sum of generation request latency.", (double)latency_us * 1e-6);
    line("barq_http_request_seconds_count", "counter", "Finished generation requests.", (double)latency_n);
    line("barq_http_active_requests", "gauge", "Generation requests in flight.", (double)active);
    line("barq_http_peak_active_requests", "gauge", "Most generation requests in flight at once.", (double)peak_active);
    line("barq_http_open_connections", "gauge", "Open client connections.", (double)connections);
    return s;
  }
};
Counters g_ctr;

// ---------------------------------------------------------------- per-client token bucket
class RateLimiter {
 public:
  bool allow(const std::string& key) {
    if (g_opt.rpm <= 0) return true;
    const double cap = g_opt.rpm, refill = cap / 60.0, t = now_s();
    std::lock_guard<std::mutex> lk(mu_);
    if (state_.size() > 65536) {  // forget clients whose bucket has refilled completely
      for (auto i = state_.begin(); i != state_.end();)
        i = (t - i->second.second) * refill + i->second.first >= cap ? state_.erase(i) : std::next(i);
    }
    auto it = state_.find(key);
    if (it == state_.end()) it = state_.emplace(key, std::make_pair(cap, t)).first;
    double& tokens = it->second.first;
    tokens = std::min(cap, tokens + (t - it->second.second) * refill);
    it->second.second = t;
    if (tokens < 1.0) return false;
    tokens -= 1.0;
    return true;
  }

 private:
  std::mutex mu_;
  std::unordered_map<std::string, std::pair<double, double>> state_;
};
RateLimiter g_limiter;

// ---------------------------------------------------------------- sockets
bool send_all(int fd, const std::string& data) {
  size_t off = 0;
  while (off < data.size()) {
    const ssize_t n = ::send(fd, data.data() + off, data.size() - off, MSG_NOSIGNAL);
    if (n < 0 && errno == EINTR) continue;
    if (n <= 0) return false;
    off += (size_t)n;
  }
  return true;
}

bool recv_exact(int fd, void* dst, size_t n) {
  char* p = static_cast<char*>(dst);
  while (n) {
    const ssize_t r = ::recv(fd, p, n, 0);
    if (r < 0 && errno == EINTR) continue;
    if (r <= 0) return false;
    p += r;
    n -= (size_t)r;
  }
  return true;
}

// ---------------------------------------------------------------- HTTP
struct Request {
  std::string method, target, path, version;
  std::vector<std::pair<std::string, std::string>> headers;  // names lower-cased
  std::string body;
  std::string header(const std::string& name) const {
    for (const auto& h : headers)
      if (h.first == name) return h.second;
    return "";
  }
};

std::string lower(std::string s) {
  for (auto& c : s) c = (char)std::tolower((unsigned char)c);
  return s;
}
std::string trim(const std::string& s) {
  size_t b = 0, e = s.size();
  while (b < e && (s[b] == ' ' || s[b] == '\t')) ++b;
  while (e > b && (s[e - 1] == ' ' || s[e - 1] == '\t' || s[e - 1] == '\r')) --e;
  return s.substr(b, e - b);
}

const char* reason_phrase(int status) {
  switch (status) {
    case 200: return "OK";
    case 204: return "No Content";
    case 400: return "Bad Request";
    case 401: return "Unauthorized";
    case 404: return "Not Found";
    case 405: return "Method Not Allowed";
    case 408: return "Request Timeout";
    case 411: return "Length Required";
    case 413: return "Payload Too Large";
    case 429: return "Too Many Requests";
    case 431: return "Request Header Fields Too Large";
    case 500: return "Internal Server Error";
    case 501: return "Not Implemented";
    case 502: return "Bad Gateway";
    case 503: return "Service Unavailable";
  }
  return "Unknown";
}

const char* kCors =
    "Access-Control-Allow-Origin: *\r\nAccess-Control-Allow-Methods: GET, POST, OPTIONS\r\n"
    "Access-Control-Allow-Headers: *\r\n";

// Buffered reader of one client connection.  read() returns 0 for a complete request, -1 when the
// peer closed (or went idle) between requests, or an HTTP status for a malformed request.
class Conn {
 public:
  explicit Conn(int fd) : fd_(fd) {}

  int read(Request& req) {
    size_t end;
    while ((end = buf_.find("\r\n\r\n")) == std::string::npos) {
      if (buf_.size() > kMaxHeaderBytes) return 431;
      if (!fill()) return buf_.empty() ? -1 : 400;
    }
    if (end > kMaxHeaderBytes) return 431;
    const std::string head = buf_.substr(0, end);
    buf_.erase(0, end + 4);
    size_t line_end = head.find("\r\n");
    const std::string first = head.substr(0, line_end);
    const size_t sp1 = first.find(' '), sp2 = first.rfind(' ');
    if (sp1 == std::string::npos || sp2 == sp1) return 400;
    req.method = first.substr(0, sp1);
    req.target = first.substr(sp1 + 1, sp2 - sp1 - 1);
    req.version = first.substr(sp2 + 1);
    if (req.version.rfind("HTTP/1.", 0) != 0 || req.target.empty()) return 400;
    req.path = req.target.substr(0, req.target.find('?'));
    req.headers.clear();
    while (line_end != std::string::npos) {
      const size_t b = line_end + 2;
      line_end = head.find("\r\n", b);
      const std::string line = head.substr(b, line_end == std::string::npos ? std::string::npos : line_end - b);
      const size_t colon = line.find(':');
      if (colon == std::string::npos || colon == 0) return 400;
      req.headers.emplace_back(lower(line.substr(0, colon)), trim(line.substr(colon + 1)));
    }
    if (!req.header("transfer-encoding").empty()) return 501;  // chunked request bodies: not accepted
    const std::string cl = req.header("content-length");
    size_t n = 0;
    if (!cl.empty()) {
      char* endp = nullptr;
      errno = 0;
      const unsigned long long v = std::strtoull(cl.c_str(), &endp, 10);
      if (errno || endp == cl.c_str() || *endp != '\0' || cl[0] == '-') return 400;
      if (v > kMaxBodyBytes) return 413;
      n = (size_t)v;
    } else if (req.method == "POST") {
      return 411;
    }
    // a client that asked to be told before it sends its body (curl does for bodies over 1 KB)
    if (buf_.size() < n && lower(req.header("expect")) == "100-continue" &&
        !send_all(fd_, "HTTP/1.1 100 Continue\r\n\r\n"))
      return -1;
    while (buf_.size() < n)
      if (!fill()) return 400;
    req.body = buf_.substr(0, n);
    buf_.erase(0, n);
    return 0;
  }

 private:
  bool fill() {
    char tmp[16384];
    for (;;) {
      const ssize_t r = ::recv(fd_, tmp, sizeof tmp, 0);
      if (r < 0 && errno == EINTR) continue;
      if (r <= 0) return false;
      buf_.append(tmp, (size_t)r);
      return true;
    }
  }
  int fd_;
  std::string buf_;
};

bool respond(int fd, int status, const std::string& ctype, const std::string& body, bool keep_alive,
             const std::string& rid) {
  std::string h = "HTTP/1.1 " + std::to_string(status) + " " + reason_phrase(status) + "\r\n";
  if (!ctype.empty()) h += "Content-Type: " + ctype + "\r\n";
  h += "Content-Length: " + std::to_string(body.size()) + "\r\n";
  h += kCors;
  if (!rid.empty()) h += "x-request-id: " + rid + "\r\n";
  h += keep_alive ? "Connection: keep-alive\r\n\r\n" : "Connection: close\r\n\r\n";
  return send_all(fd, h + body);
}

std::string error_body(const std::string& msg, const std::string& kind) {
  Value e = Value::object(), err = Value::object();
  err.set("message", Value::string(msg));
  err.set("type", Value::string(kind));
  e.set("error", err);
  return barqjson::dump(e);
}

const char* error_kind(int status) {
  switch (status) {
    case 401: return "authentication_error";
    case 404: return "not_found_error";
    case 429: return "rate_limit_error";
    case 502: return "engine_unavailable_error";
    case 503: return "overloaded_error";
  }
  return status >= 500 ? "server_error" : "invalid_request_error";
}

// ---------------------------------------------------------------- engine pool
// Several engine processes (e.g. one per GPU) can serve behind one front end: each request goes to
// the engine with the fewest requests in flight among those that accept connections; an engine
// whose socket refuses is skipped for a few seconds and the request fails over to the next one.
struct EnginePool {
  static constexpr int kMax = 64;
  std::atomic<int> active[kMax];
  std::atomic<double> down_until[kMax];
  EnginePool() {
    for (int i = 0; i < kMax; ++i) {
      active[i] = 0;
      down_until[i] = 0.0;
    }
  }
  // Engine indices in the order to try: fewest in flight first, engines marked down last.
  std::vector<int> order() {
    const int n = (int)g_opt.sockets.size();
    const double t = now_s();
    std::vector<int> idx(n);
    for (int i = 0; i < n; ++i) idx[i] = i;
    std::stable_sort(idx.begin(), idx.end(), [&](int a, int b) {
      const bool da = down_until[a] > t, db = down_until[b] > t;
      if (da != db) return !da;
      return active[a].load() < active[b].load();
    });
    return idx;
  }
};
EnginePool g_pool;

// ---------------------------------------------------------------- engine link (UDS frames)
class EngineLink {
 public:
  ~EngineLink() { close(); }

  // Connects to the least busy engine that answers (or to engine `only` when it is >= 0).
  bool open(std::string& err, int only = -1) {
    std::vector<int> order = only >= 0 ? std::vector<int>{only} : g_pool.order();
    for (int i : order) {
      if (connect_to(i, err)) {
        idx_ = i;
        ++g_pool.active[i];
        return true;
      }
      g_pool.down_until[i] = now_s() + 5.0;
    }
    return false;
  }
  int engine() const { return idx_; }
  bool send(const Value& frame) {
    const std::string body = barqjson::dump(frame);
    const uint32_t n = (uint32_t)body.size();
    const unsigned char head[4] = {(unsigned char)(n >> 24), (unsigned char)(n >> 16), (unsigned char)(n >> 8),
                                   (unsigned char)n};
    return send_all(fd_, std::string(reinterpret_cast<const char*>(head), 4) + body);
  }
  // One frame, or false with `err` set (closed, timed out, oversized or not a JSON object).
  bool next(Value& frame, std::string& err) {
    unsigned char head[4];
    if (!recv_exact(fd_, head, 4)) {
      err = "engine closed the stream";
      return false;
    }
    const uint32_t n = ((uint32_t)head[0] << 24) | ((uint32_t)head[1] << 16) | ((uint32_t)head[2] << 8) | head[3];
    if (n > kMaxFrame) {
      err = "engine frame too large";
      return false;
    }
    std::string body(n, '\0');
    if (n && !recv_exact(fd_, &body[0], n)) {
      err = "engine closed the stream";
      return false;
    }
    try {
      frame = barqjson::parse(body);
    } catch (const std::exception& e) {
      err = std::string("bad engine frame: ") + e.what();
      return false;
    }
    if (!frame.is_object()) {
      err = "bad engine frame: not an object";
      return false;
    }
    return true;
  }
  void close() {
    if (fd_ >= 0) ::close(fd_);
    fd_ = -1;
    if (idx_ >= 0) --g_pool.active[idx_];
    idx_ = -1;
  }

 private:
  bool connect_to(int i, std::string& err) {
    const std::string& path = g_opt.sockets[i];
    fd_ = ::socket(AF_UNIX, SOCK_STREAM, 0);
    if (fd_ < 0) {
      err = std::strerror(errno);
      return false;
    }
    sockaddr_un addr{};
    addr.sun_family = AF_UNIX;
    if (path.size() >= sizeof(addr.sun_path)) {
      err = "socket path too long";
      ::close(fd_);
      fd_ = -1;
      return false;
    }
    std::memcpy(addr.sun_path, path.c_str(), path.size() + 1);
    if (::connect(fd_, reinterpret_cast<sockaddr*>(&addr), sizeof(addr)) != 0) {
      err = std::string("cannot connect to ") + path + ": " + std::strerror(errno);
      ::close(fd_);
      fd_ = -1;
      return false;
    }
    timeval tv{};
    tv.tv_sec = g_opt.engine_timeout_s;
    setsockopt(fd_, SOL_SOCKET, SO_RCVTIMEO, &tv, sizeof tv);
    return true;
  }
  int fd_ = -1, idx_ = -1;
};

// One-frame engine query ({"health": true} -> {"healthy", "last_error", "kv_usage"};
// {"metrics": true} -> {"prometheus"}), or a null value when the engine socket does not answer.
Value engine_query(const char* what, int engine) {
  EngineLink l;
  std::string err;
  if (!l.open(err, engine)) return Value();
  Value req = Value::object(), fr;
  req.set("id", Value::string(what));
  req.set(what, Value::boolean(true));
  if (!l.send(req) || !l.next(fr, err)) return Value();
  return fr;
}

// True when the client has closed its side (checked between streamed pieces of a non-streamed
// response, so that a client that gave up stops its generation).
bool client_gone(int fd) {
  pollfd p{fd, POLLIN | POLLRDHUP, 0};
  if (::poll(&p, 1, 0) <= 0) return false;
  if (p.revents & (POLLRDHUP | POLLHUP | POLLERR)) return true;
  char c;
  return ::recv(fd, &c, 1, MSG_PEEK | MSG_DONTWAIT) == 0;
}

// ---------------------------------------------------------------- one generation
struct Gen {
  std::string text;
  std::string finish = "stop";
  Value tool_call;  // {"name", "arguments"} when the engine recognized a call of one of the tools
  std::vector<Value> lps;  // per-token logprob entries of the text returned (non-streamed calls)
  long prompt_tokens = 0, completion_tokens = 0;
  int status = 200;  // non-200: `error` says why
  std::string error;
};

// Stop strings: returns the earliest match position in `text`, or npos.
size_t find_stop(const std::string& text, const std::vector<std::string>& stops, size_t from) {
  size_t best = std::string::npos;
  for (const auto& s : stops) {
    if (s.empty()) continue;
    const size_t b = from > s.size() ? from - s.size() : 0;
    const size_t p = text.find(s, b);
    if (p != std::string::npos && p < best) best = p;
  }
  return best;
}
// Length of the longest suffix of `text` that is a proper prefix of some stop string.
size_t held_suffix(const std::string& text, const std::vector<std::string>& stops) {
  size_t hold = 0;
  for (const auto& s : stops)
    for (size_t k = std::min(s.size() - (s.empty() ? 0 : 1), text.size()); k > hold; --k)
      if (text.compare(text.size() - k, k, s, 0, k) == 0) {
        hold = k;
        break;
      }
  return hold;
}

int engine_error_status(const std::string& msg) {
  if (msg == "queue full" || msg.find("overloaded") != std::string::npos) return 503;
  if (msg.rfind("bad request", 0) == 0 || msg.find("exceeds max_model_len") != std::string::npos) return 400;
  return 500;
}

// Runs one request on the engine.  `on_first` is called once before the first delta (or not at all
// when the engine refuses the request), `on_delta` with every piece of text that can no longer be
// part of a stop string; either returning false (client gone) ends the generation early.
Gen generate(const Value& uds_req, const std::vector<std::string>& stops, const std::function<bool()>& on_first,
             const std::function<bool(const std::string&, std::vector<Value>&)>& on_delta) {
  Gen g;
  EngineLink link;
  std::string err;
  const double t0 = now_s();
  if (!link.open(err)) {
    g.status = 502;
    g.error = "engine unavailable: " + err;
    return g;
  }
  if (!link.send(uds_req)) {
    g.status = 502;
    g.error = "engine unavailable: send failed";
    return g;
  }
  size_t sent = 0;  // bytes of g.text already handed to on_delta
  bool first = true;
  std::vector<Value> pend;  // logprob entries of tokens whose text has not been handed out yet
  auto emit = [&](const std::string& d) {
    for (auto& e : pend) g.lps.push_back(e);
    const bool ok = on_delta(d, pend);
    pend.clear();
    return ok;
  };
  for (;;) {
    Value fr;
    if (!link.next(fr, err)) {
      g.status = 500;
      g.error = err;
      return g;
    }
    const Value* e = fr.get("error");
    const Value* done = fr.get("done");
    const bool is_done = done && done->type == Value::kBool && done->b;
    if (e && e->is_string()) {
      g.status = engine_error_status(e->str);
      g.error = e->str;
      return g;
    }
    const Value* t = fr.get("text");
    const std::string piece = t && t->is_string() ? t->str : "";
    if (const Value* lp = fr.get("logprobs"); lp && lp->is_array())
      for (const auto& e : lp->arr) pend.push_back(e);
    if (const Value* n = fr.get("tokens_generated"); n && n->is_number()) g.completion_tokens = (long)n->num;
    if (first && (!piece.empty() || is_done)) {
      first = false;
      if (!piece.empty() || g.completion_tokens > 0) {
        g_ctr.ttft_us += (uint64_t)((now_s() - t0) * 1e6);
        ++g_ctr.ttft_n;
      }
      if (!on_first()) return g;
    }
    const size_t before = g.text.size();
    g.text += piece;
    const size_t hit = stops.empty() ? std::string::npos : find_stop(g.text, stops, before);
    if (hit != std::string::npos) {
      g.text.resize(hit);
      g.finish = "stop";
      if (hit > sent) emit(g.text.substr(sent));
      return g;  // closing the link aborts the request in the engine
    }
    if (is_done) {
      if (const Value* p = fr.get("prompt_tokens"); p && p->is_number()) g.prompt_tokens = (long)p->num;
      if (const Value* f = fr.get("finish_reason"); f && f->is_string()) g.finish = f->str;
      if (const Value* tc = fr.get("tool_call"); tc && tc->is_object()) g.tool_call = *tc;
      if (g.text.size() > sent || !pend.empty()) emit(g.text.substr(sent));
      return g;
    }
    const size_t safe = g.text.size() - (stops.empty() ? 0 : held_suffix(g.text, stops));
    if (safe > sent) {
      if (!emit(g.text.substr(sent, safe - sent))) return g;
      sent = safe;
    }
  }
}

// ---------------------------------------------------------------- request translation
struct Call {
  std::string kind;  // "text", "chat", "resp"
  Value uds;         // the engine request
  std::vector<std::string> stops;
  bool stream = false, include_usage = false, tools = false, logprobs = false;
  std::vector<Value> prompts;  // a batch of prompts (completions), else empty
  int n = 1;
  std::string model;
};

[[noreturn]] void bad(const std::string& msg) { throw std::invalid_argument(msg); }

Call translate(const std::string& kind, const Value& body, const std::string& rid) {
  if (!body.is_object()) bad("request body must be a JSON object");
  Call c;
  c.kind = kind;
  c.uds = Value::object();
  c.uds.set("id", Value::string(rid));
  const Value* model = body.get("model");
  c.model = model && model->is_string() && !model->str.empty() ? model->str : g_opt.model_id;
  auto messages = [&](const Value& m) {
    if (!m.is_array() || m.arr.empty()) bad("messages must be a non-empty list");
    for (const auto& x : m.arr)
      if (!x.is_object() || !x.get("content")) bad("each message needs role and content");
    c.uds.set("messages", m);
  };
  if (kind == "text") {
    const Value* p = body.get("prompt");
    bool ok = p && p->is_string(), ids = false, batch = false;
    if (p && p->is_array() && !p->arr.empty()) {
      ids = batch = true;
      for (const auto& t : p->arr) {
        ids = ids && t.is_integer();
        bool one = t.is_string();
        if (t.is_array() && !t.arr.empty()) {
          one = true;
          for (const auto& x : t.arr) one = one && x.is_integer();
        }
        batch = batch && one;
      }
      ok = ids || batch;
    }
    if (!ok) bad("prompt must be a string, a list of strings or token id list(s)");
    if (batch && !ids) {  // a batch of prompts: n choices for each, indexed prompt-major
      c.prompts = p->arr;
      c.uds.set("prompt", p->arr[0]);
    } else {
      c.uds.set("prompt", *p);
    }
  } else if (kind == "chat") {
    const Value* m = body.get("messages");
    if (!m) bad("messages must be a non-empty list");
    messages(*m);
    if (const Value* t = body.get("tools"); t && !t->is_null()) {
      if (!t->is_array()) bad("tools must be a list");
      c.uds.set("tools", *t);
      c.tools = !t->arr.empty();
      if (const Value* tc = body.get("tool_choice"); tc && !tc->is_null()) c.uds.set("tool_choice", *tc);
    }
  } else {
    if (const Value* m = body.get("messages"); m && !m->is_null()) {
      messages(*m);
    } else {
      const Value* in = body.get("input");
      if (!in || in->is_null()) in = body.get("prompt");
      if (in && in->is_string()) c.uds.set("prompt", *in);
      else if (in && in->is_array()) messages(*in);
      else bad("input (or prompt / messages) is required");
    }
  }
  const Value* mt = body.get(kind == "resp" ? "max_output_tokens" : "max_tokens");
  if (!mt || mt->is_null()) mt = body.get("max_tokens");
  if (mt && !mt->is_null()) {
    if (!mt->is_integer() || mt->num < 1) bad("max_tokens must be >= 1");
    c.uds.set("max_tokens", *mt);
  }
  static const char* kForward[] = {"temperature", "top_k", "top_p", "min_p", "seed", "repetition_penalty",
                                   "frequency_penalty", "presence_penalty", "response_format", "grammar"};
  for (const char* k : kForward) {
    const Value* v = body.get(k);
    if (!v || v->is_null()) continue;
    const bool numeric = std::strcmp(k, "response_format") != 0 && std::strcmp(k, "grammar") != 0;
    if (numeric && !v->is_number()) bad(std::string(k) + " must be a number");
    c.uds.set(k, *v);
  }
  if (const Value* lp = body.get("logprobs"); lp && !lp->is_null()) {
    if (lp->type == Value::kBool) c.logprobs = lp->b;
    else if (lp->is_integer() && lp->num >= 0 && lp->num <= 20) c.logprobs = true;
    else bad("logprobs must be a boolean or an integer (0..20)");
    c.uds.set("logprobs", *lp);
    if (const Value* tl = body.get("top_logprobs"); tl && !tl->is_null()) {
      if (!tl->is_integer() || tl->num < 0 || tl->num > 20) bad("top_logprobs must be between 0 and 20");
      c.uds.set("top_logprobs", *tl);
    }
  }
  if (const Value* s = body.get("stop"); s && !s->is_null()) {
    if (s->is_string()) {
      c.stops.push_back(s->str);
    } else if (s->is_array()) {
      for (const auto& x : s->arr) {
        if (!x.is_string()) bad("stop must be a string or a list of strings");
        c.stops.push_back(x.str);
      }
    } else {
      bad("stop must be a string or a list of strings");
    }
  }
  if (const Value* n = body.get("n"); n && !n->is_null()) {
    if (!n->is_integer() || n->num < 1 || n->num > 16) bad("n must be between 1 and 16");
    c.n = (int)n->num;
  }
  if (const Value* s = body.get("stream"); s && s->type == Value::kBool) c.stream = s->b;
  if (c.stream && c.n > 1) bad("n > 1 is not supported with stream");
  if (c.stream && c.tools) bad("stream with tools is not supported; send stream=false");
  if (c.stream && !c.prompts.empty()) bad("a batch of prompts is not supported with stream");
  if (const Value* so = body.get("stream_options"); so && so->is_object())
    if (const Value* iu = so->get("include_usage"); iu && iu->type == Value::kBool) c.include_usage = iu->b;
  return c;
}

std::string make_id(const std::string& kind) {
  static std::atomic<uint64_t> seq{0};
  const char* prefix = kind == "text" ? "cmpl" : kind == "chat" ? "chatcmpl" : "resp";
  return std::string(prefix) + "-" + std::to_string((long long)std::time(nullptr)) + std::to_string(++seq % 100000);
}

Value usage(long p, long c) {
  Value u = Value::object();
  u.set("prompt_tokens", Value::number((double)p));
  u.set("completion_tokens", Value::number((double)c));
  u.set("total_tokens", Value::number((double)(p + c)));
  return u;
}

// OpenAI logprob objects from the engine's entries {token, bytes, logprob, top: [...]}.
Value lp_chat(const std::vector<Value>& ents) {
  Value content = Value::array();
  for (const auto& e : ents) {
    Value o = Value::object(), tops = Value::array();
    for (const char* k : {"token", "logprob", "bytes"})
      if (const Value* v = e.get(k)) o.set(k, *v);
    if (const Value* t = e.get("top"); t && t->is_array())
      for (const auto& a : t->arr) {
        Value x = Value::object();
        for (const char* k : {"token", "logprob", "bytes"})
          if (const Value* v = a.get(k)) x.set(k, *v);
        tops.push(x);
      }
    o.set("top_logprobs", tops);
    content.push(o);
  }
  Value r = Value::object();
  r.set("content", content);
  return r;
}

Value lp_text(const std::vector<Value>& ents, size_t& offset) {
  Value toks = Value::array(), lps = Value::array(), tops = Value::array(), offs = Value::array();
  bool any_top = false;
  for (const auto& e : ents) {
    const Value* t = e.get("token");
    const std::string tok = t && t->is_string() ? t->str : "";
    toks.push(Value::string(tok));
    const Value* lp = e.get("logprob");
    lps.push(lp ? *lp : Value());
    const Value* top = e.get("top");
    if (top && top->is_array() && !top->arr.empty()) {
      any_top = true;
      Value m = Value::object();
      for (const auto& a : top->arr) {
        const Value* at = a.get("token");
        const Value* al = a.get("logprob");
        m.set(at && at->is_string() ? at->str : "", al ? *al : Value());
      }
      tops.push(m);
    } else {
      tops.push(Value());
    }
    offs.push(Value::number((double)offset));
    offset += tok.size();
  }
  Value r = Value::object();
  r.set("tokens", toks);
  r.set("token_logprobs", lps);
  r.set("top_logprobs", any_top ? tops : Value());
  r.set("text_offset", offs);
  return r;
}

Value chunk(const Call& c, const std::string& id, long created, const std::string* delta, const std::string* finish,
            bool role) {
  Value o = Value::object();
  o.set("id", Value::string(id));
  o.set("object", Value::string(c.kind == "text" ? "text_completion.chunk"
                                : c.kind == "chat" ? "chat.completion.chunk" : "response.chunk"));
  o.set("created", Value::number((double)created));
  o.set("model", Value::string(c.model));
  if (c.kind == "resp") {
    o.set("output", Value::string(delta ? *delta : ""));
    return o;
  }
  Value ch = Value::object();
  ch.set("index", Value::number(0));
  if (c.kind == "text") {
    ch.set("text", Value::string(delta ? *delta : ""));
  } else {
    Value d = Value::object();
    if (role) d.set("role", Value::string("assistant"));
    if (delta) d.set("content", Value::string(*delta));
    ch.set("delta", d);
  }
  ch.set("finish_reason", finish ? Value::string(*finish) : Value());
  Value arr = Value::array();
  arr.push(ch);
  o.set("choices", arr);
  return o;
}

// ---------------------------------------------------------------- handlers
struct Outcome {
  int status = 200;
  bool close = false;  // the connection cannot be reused (a streamed response was sent)
};

Outcome finish_error(int fd, int status, const std::string& msg, bool keep, const std::string& rid) {
  respond(fd, status, "application/json", error_body(msg, error_kind(status)), keep, rid);
  return Outcome{status, !keep};
}

Outcome generate_route(int fd, const std::string& kind, const Request& req, bool keep, const std::string& rid) {
  Value body;
  try {
    body = barqjson::parse(req.body);
  } catch (const std::exception&) {
    return finish_error(fd, 400, "request body is not valid JSON", keep, rid);
  }
  Call c;
  try {
    c = translate(kind, body, rid);
  } catch (const std::invalid_argument& e) {
    return finish_error(fd, 400, e.what(), keep, rid);
  }
  const std::string id = make_id(kind);
  const long created = (long)std::time(nullptr);
  const double t0 = now_s();
  g_ctr.begin();
  struct ActiveGuard {
    double t0;
    ~ActiveGuard() {
      --g_ctr.active;
      g_ctr.latency_us += (uint64_t)((now_s() - t0) * 1e6);
      ++g_ctr.latency_n;
    }
  } guard{t0};

  if (c.stream) {
    // HTTP/1.1 clients get the event stream chunk-encoded, so the connection stays reusable;
    // HTTP/1.0 clients get it close-delimited
    const bool chunked = req.version == "HTTP/1.1";
    bool headers_sent = false, client_ok = true;
    auto put = [&](const std::string& data) {
      if (!chunked) return send_all(fd, data);
      char len[24];
      std::snprintf(len, sizeof len, "%zx\r\n", data.size());
      return send_all(fd, len + data + "\r\n");
    };
    auto send_event = [&](const Value& v) {
      client_ok = client_ok && put("data: " + barqjson::dump(v) + "\n\n");
      return client_ok;
    };
    auto on_first = [&]() {
      std::string h = "HTTP/1.1 200 OK\r\nContent-Type: text/event-stream\r\nCache-Control: no-cache\r\n";
      h += kCors;
      h += "x-request-id: " + rid + "\r\n";
      h += chunked ? std::string("Transfer-Encoding: chunked\r\n") + (keep ? "Connection: keep-alive\r\n\r\n"
                                                                         : "Connection: close\r\n\r\n")
                   : "Connection: close\r\n\r\n";
      headers_sent = true;
      client_ok = send_all(fd, h);
      if (client_ok && kind == "chat") send_event(chunk(c, id, created, nullptr, nullptr, true));
      return client_ok;
    };
    size_t offset = 0;
    auto on_delta = [&](const std::string& d, std::vector<Value>& ents) {
      Value ev = chunk(c, id, created, &d, nullptr, false);
      if (c.logprobs && kind != "resp")
        for (auto& kv : ev.obj)
          if (kv.first == "choices") kv.second.arr[0].set("logprobs", kind == "chat" ? lp_chat(ents) : lp_text(ents, offset));
      return send_event(ev);
    };
    Gen g = generate(c.uds, c.stops, on_first, on_delta);
    if (!headers_sent) {
      if (g.status != 200) return finish_error(fd, g.status, g.error, keep, rid);
      on_first();  // an empty generation still gets its stream
    }
    if (g.status != 200) {  // failed after the stream started: an error event, then the end marker
      client_ok = client_ok && put("data: " + error_body(g.error, error_kind(g.status)) + "\n\n");
    } else if (client_ok) {
      if (kind != "resp") send_event(chunk(c, id, created, nullptr, &g.finish, false));
      if (c.include_usage) {
        Value u = Value::object();
        u.set("id", Value::string(id));
        u.set("object", Value::string(kind == "chat" ? "chat.completion.chunk" : "text_completion.chunk"));
        u.set("created", Value::number((double)created));
        u.set("model", Value::string(c.model));
        u.set("choices", Value::array());
        u.set("usage", usage(g.prompt_tokens, g.completion_tokens));
        send_event(u);
      }
      g_ctr.prompt_tokens += (uint64_t)g.prompt_tokens;
      g_ctr.completion_tokens += (uint64_t)g.completion_tokens;
    }
    if (client_ok) client_ok = put("data: [DONE]\n\n");
    if (client_ok && chunked) client_ok = send_all(fd, "0\r\n\r\n");  // last chunk
    return Outcome{g.status == 200 ? 200 : g.status, !(chunked && keep && client_ok)};
  }

  // the n choices (of every prompt of a batch) run as concurrent engine requests (continuous
  // batching serves them together); choice index = prompt * n + i
  const int n_prompts = c.prompts.empty() ? 1 : (int)c.prompts.size();
  std::vector<Gen> outs(n_prompts * c.n);
  std::vector<std::thread> workers;
  for (int q = 0; q < n_prompts * c.n; ++q) {
    const int i = q % c.n;
    Value r = c.uds;
    if (!c.prompts.empty()) r.set("prompt", c.prompts[q / c.n]);
    if (q > 0) r.set("id", Value::string(rid + "-" + std::to_string(q)));
    if (i > 0) {  // choice i samples with its own seed (a 0 seed already differs per request)
      const Value* s = r.get("seed");
      if (s && s->is_number() && s->num != 0) r.set("seed", Value::number(s->num + i));
    }
    auto run = [&outs, &c, q, fd](Value req) {
      // a client that has gone away stops the generation (closing the link aborts it in the engine)
      outs[q] = generate(req, c.stops, [] { return true; },
                         [fd](const std::string&, std::vector<Value>&) { return !client_gone(fd); });
    };
    if (q + 1 < n_prompts * c.n) workers.emplace_back(run, std::move(r));
    else run(std::move(r));
  }
  for (auto& w : workers) w.join();
  long p_tok = 0, c_tok = 0;
  for (size_t q = 0; q < outs.size(); ++q) {
    const Gen& g = outs[q];
    if (g.status != 200) return finish_error(fd, g.status, g.error, keep, rid);
    if ((int)q % c.n == 0) p_tok += g.prompt_tokens;  // each prompt counted once
    c_tok += g.completion_tokens;
  }
  g_ctr.prompt_tokens += (uint64_t)p_tok;
  g_ctr.completion_tokens += (uint64_t)c_tok;
  Value o = Value::object();
  o.set("id", Value::string(id));
  o.set("object", Value::string(kind == "text" ? "text_completion" : kind == "chat" ? "chat.completion" : "response"));
  o.set("created", Value::number((double)created));
  o.set("model", Value::string(c.model));
  if (kind == "resp") {
    o.set("output", Value::string(outs[0].text));
  } else {
    Value arr = Value::array();
    for (size_t i = 0; i < outs.size(); ++i) {
      Value ch = Value::object();
      ch.set("index", Value::number((double)i));
      if (kind == "text") {
        ch.set("text", Value::string(outs[i].text));
      } else if (outs[i].tool_call.is_object()) {  // the reply is a call of one of the tools
        Value m = Value::object(), calls = Value::array(), call = Value::object(), fn = Value::object();
        const Value* name = outs[i].tool_call.get("name");
        const Value* args = outs[i].tool_call.get("arguments");
        fn.set("name", name ? *name : Value::string(""));
        fn.set("arguments", Value::string(args ? barqjson::dump(*args) : "{}"));
        call.set("id", Value::string("call_" + id + "_" + std::to_string(i)));
        call.set("type", Value::string("function"));
        call.set("function", fn);
        calls.push(call);
        m.set("role", Value::string("assistant"));
        m.set("content", Value());
        m.set("tool_calls", calls);
        ch.set("message", m);
      } else {
        Value m = Value::object();
        m.set("role", Value::string("assistant"));
        m.set("content", Value::string(outs[i].text));
        ch.set("message", m);
      }
      ch.set("finish_reason", Value::string(outs[i].finish));
      if (c.logprobs) {
        size_t off = 0;
        ch.set("logprobs", kind == "chat" ? lp_chat(outs[i].lps) : lp_text(outs[i].lps, off));
      } else {
        ch.set("logprobs", Value());
      }
      arr.push(ch);
    }
    o.set("choices", arr);
  }
  o.set("usage", usage(p_tok, c_tok));
  respond(fd, 200, "application/json", barqjson::dump(o), keep, rid);
  return Outcome{200, !keep};
}

Outcome embeddings_route(int fd, const Request& req, bool keep, const std::string& rid) {
  Value body;
  try {
    body = barqjson::parse(req.body);
  } catch (const std::exception&) {
    return finish_error(fd, 400, "request body is not valid JSON", keep, rid);
  }
  const Value* in = body.is_object() ? body.get("input") : nullptr;
  if (!in || !(in->is_string() || (in->is_array() && !in->arr.empty())))
    return finish_error(fd, 400, "input must be a string, a list of strings or token-id list(s)", keep, rid);
  Value r = Value::object();
  r.set("id", Value::string(rid));
  r.set("embeddings", *in);
  EngineLink link;
  std::string err;
  if (!link.open(err)) return finish_error(fd, 502, "engine unavailable: " + err, keep, rid);
  Value fr;
  if (!link.send(r) || !link.next(fr, err)) return finish_error(fd, 500, err.empty() ? "send failed" : err, keep, rid);
  if (const Value* e = fr.get("error"); e && e->is_string()) return finish_error(fd, engine_error_status(e->str), e->str, keep, rid);
  const Value* vecs = fr.get("embeddings");
  if (!vecs || !vecs->is_array()) return finish_error(fd, 500, "engine frame without embeddings", keep, rid);
  Value o = Value::object(), data = Value::array();
  for (size_t i = 0; i < vecs->arr.size(); ++i) {
    Value d = Value::object();
    d.set("object", Value::string("embedding"));
    d.set("index", Value::number((double)i));
    d.set("embedding", vecs->arr[i]);
    data.push(d);
  }
  const Value* model = body.get("model");
  const Value* pt = fr.get("prompt_tokens");
  const double n = pt && pt->is_number() ? pt->num : 0;
  Value u = Value::object();
  u.set("prompt_tokens", Value::number(n));
  u.set("total_tokens", Value::number(n));
  o.set("object", Value::string("list"));
  o.set("model", model && model->is_string() ? *model : Value::string(g_opt.model_id));
  o.set("data", data);
  o.set("usage", u);
  respond(fd, 200, "application/json", barqjson::dump(o), keep, rid);
  return Outcome{200, !keep};
}

// llama.cpp-style /tokenize ({"content", "add_special"} -> {"tokens"}) and /detokenize
// ({"tokens"} -> {"content"}), answered by the engine's tokenizer.
Outcome tokenize_route(int fd, const Request& req, bool keep, const std::string& rid, bool detok) {
  Value body;
  try {
    body = barqjson::parse(req.body);
  } catch (const std::exception&) {
    return finish_error(fd, 400, "request body is not valid JSON", keep, rid);
  }
  Value r = Value::object();
  r.set("id", Value::string(rid));
  const Value* in = body.is_object() ? body.get(detok ? "tokens" : "content") : nullptr;
  if (!in || (detok ? !in->is_array() : !in->is_string()))
    return finish_error(fd, 400, detok ? "tokens must be a list of token ids" : "content must be a string", keep, rid);
  r.set(detok ? "detokenize" : "tokenize", *in);
  if (!detok)
    if (const Value* a = body.get("add_special"); a && a->type == Value::kBool) r.set("add_special", *a);
  EngineLink link;
  std::string err;
  Value fr;
  if (!link.open(err)) return finish_error(fd, 502, "engine unavailable: " + err, keep, rid);
  if (!link.send(r) || !link.next(fr, err)) return finish_error(fd, 500, err.empty() ? "send failed" : err, keep, rid);
  if (const Value* e = fr.get("error"); e && e->is_string()) return finish_error(fd, engine_error_status(e->str), e->str, keep, rid);
  Value o = Value::object();
  const Value* v = fr.get(detok ? "content" : "tokens");
  o.set(detok ? "content" : "tokens", v ? *v : Value());
  respond(fd, 200, "application/json", barqjson::dump(o), keep, rid);
  return Outcome{200, !keep};
}

std::string request_id(const Request& req) {
  std::string rid = req.header("x-request-id");
  bool clean = !rid.empty() && rid.size() <= 128;
  for (const char ch : rid) clean = clean && (std::isalnum((unsigned char)ch) || ch == '-' || ch == '_' || ch == '.');
  if (clean) return rid;
  static std::atomic<uint64_t> seq{0};
  thread_local uint64_t salt = (uint64_t)std::chrono::steady_clock::now().time_since_epoch().count();
  char buf[24];
  std::snprintf(buf, sizeof buf, "%016llx", (unsigned long long)((salt * 0x9E3779B97F4A7C15ull) ^ ++seq));
  return buf;
}

// Constant-time comparison of the Authorization header with "Bearer <key>".
bool authorized(const Request& req) {
  if (g_opt.api_key.empty()) return true;
  const std::string want = "Bearer " + g_opt.api_key, got = req.header("authorization");
  unsigned diff = (unsigned)(want.size() ^ got.size());
  for (size_t i = 0; i < want.size(); ++i) diff |= (unsigned char)want[i] ^ (unsigned char)(i < got.size() ? got[i] : 0);
  return diff == 0;
}

Outcome dispatch(int fd, const Request& req, const std::string& client, bool keep) {
  const std::string rid = request_id(req);
  if (req.method == "OPTIONS") {
    respond(fd, 204, "", "", keep, rid);
    return Outcome{204, !keep};
  }
  const std::string& p = req.path;
  if (p.rfind("/v1/", 0) == 0 && !authorized(req))
    return finish_error(fd, 401, "missing or invalid API key", keep, rid);
  if (req.method == "GET") {
    if (p == "/") {
      Value o = Value::object(), eps = Value::array();
      o.set("object", Value::string("server.info"));
      o.set("model", Value::string(g_opt.model_id));
      o.set("front_end", Value::string("barq-http"));
      for (const char* e : {"/v1/models", "/v1/responses", "/v1/completions", "/v1/chat/completions",
                            "/v1/embeddings", "/tokenize", "/detokenize", "/health", "/metrics"})
        eps.push(Value::string(e));
      o.set("endpoints", eps);
      respond(fd, 200, "application/json", barqjson::dump(o), keep, rid);
      return Outcome{200, !keep};
    }
    if (p == "/v1/models") {
      Value o = Value::object(), data = Value::array(), m = Value::object();
      m.set("id", Value::string(g_opt.model_id));
      m.set("object", Value::string("model"));
      m.set("created", Value::number((double)std::time(nullptr)));
      m.set("owned_by", Value::string("barq"));
      data.push(m);
      o.set("object", Value::string("list"));
      o.set("data", data);
      respond(fd, 200, "application/json", barqjson::dump(o), keep, rid);
      return Outcome{200, !keep};
    }
    if (p.rfind("/v1/models/", 0) == 0) {  // retrieve one model
      const std::string name = p.substr(11);
      if (name != g_opt.model_id) return finish_error(fd, 404, "model '" + name + "' not found", keep, rid);
      Value m = Value::object();
      m.set("id", Value::string(g_opt.model_id));
      m.set("object", Value::string("model"));
      m.set("created", Value::number((double)std::time(nullptr)));
      m.set("owned_by", Value::string("barq"));
      respond(fd, 200, "application/json", barqjson::dump(m), keep, rid);
      return Outcome{200, !keep};
    }
    if (p == "/health") {  // ok while any engine is up and healthy
      Value o = Value::object(), engines = Value::array();
      int n_ok = 0, n_up = 0;
      for (int i = 0; i < (int)g_opt.sockets.size(); ++i) {
        const Value h = engine_query("health", i);
        const Value* healthy = h.get("healthy");
        const bool up = h.is_object(), ok = up && (!healthy || healthy->type != Value::kBool || healthy->b);
        n_up += up;
        n_ok += ok;
        Value e = Value::object();
        e.set("socket", Value::string(g_opt.sockets[i]));
        e.set("status", Value::string(!up ? "unreachable" : ok ? "ok" : "degraded"));
        e.set("active_requests", Value::number((double)g_pool.active[i].load()));
        for (const char* k : {"kv_usage", "last_error"})
          if (const Value* v = h.get(k)) e.set(k, *v);
        engines.push(e);
      }
      o.set("status", Value::string(n_ok ? "ok" : n_up ? "degraded" : "engine_unreachable"));
      o.set("active_requests", Value::number((double)g_ctr.active));
      const Value first = engines.arr.empty() ? Value() : engines.arr[0];
      for (const char* k : {"kv_usage", "last_error"})
        if (const Value* v = first.get(k)) o.set(k, *v);
      o.set("engines", engines);
      respond(fd, n_ok ? 200 : 503, "application/json", barqjson::dump(o), keep, rid);
      return Outcome{n_ok ? 200 : 503, !keep};
    }
    if (p == "/metrics") {  // this front end's counters, then every engine's own (one scrape target)
      std::string text = g_ctr.prometheus();
      const int n = (int)g_opt.sockets.size();
      for (int i = 0; i < n; ++i) {
        const Value m = engine_query("metrics", i);
        const Value* t = m.get("prometheus");
        if (!t || !t->is_string()) continue;
        if (n == 1) {
          text += t->str;
          continue;
        }
        // several engines: label every sample with its engine, HELP / TYPE lines once
        size_t b = 0;
        while (b < t->str.size()) {
          size_t e = t->str.find('\n', b);
          if (e == std::string::npos) e = t->str.size();
          std::string line = t->str.substr(b, e - b);
          b = e + 1;
          if (line.empty()) continue;
          if (line[0] == '#') {
            if (i == 0) text += line + "\n";
            continue;
          }
          const size_t brace = line.find('{'), sp = line.find(' ');
          const std::string lab = "engine=\"" + std::to_string(i) + "\"";
          if (brace != std::string::npos && brace < sp)
            line.insert(brace + 1, lab + ",");
          else if (sp != std::string::npos)
            line.insert(sp, "{" + lab + "}");
          text += line + "\n";
        }
      }
      respond(fd, 200, "text/plain; version=0.0.4", text, keep, rid);
      return Outcome{200, !keep};
    }
  }
  if (p == "/tokenize" || p == "/detokenize") {
    if (req.method != "POST") return finish_error(fd, 405, "use POST for " + p, keep, rid);
    return tokenize_route(fd, req, keep, rid, p == "/detokenize");
  }
  if (p == "/v1/embeddings") {
    if (req.method != "POST") return finish_error(fd, 405, "use POST for " + p, keep, rid);
    if (!g_limiter.allow(client)) {
      ++g_ctr.rate_limited;
      return finish_error(fd, 429, "rate limit exceeded; retry later", keep, rid);
    }
    return embeddings_route(fd, req, keep, rid);
  }
  static const std::map<std::string, std::string> kRoutes = {
      {"/v1/completions", "text"}, {"/v1/chat/completions", "chat"}, {"/v1/responses", "resp"}};
  const auto it = kRoutes.find(p);
  if (it != kRoutes.end()) {
    if (req.method != "POST") return finish_error(fd, 405, "use POST for " + p, keep, rid);
    ++g_ctr.requests;
    if (!g_limiter.allow(client)) {
      ++g_ctr.rate_limited;
      return finish_error(fd, 429, "rate limit exceeded; retry later", keep, rid);
    }
    return generate_route(fd, it->second, req, keep, rid);
  }
  return finish_error(fd, 404,
                      "route not found; try /v1/models, /v1/responses, /v1/completions or /v1/chat/completions",
                      keep, rid);
}

void log_line(const Request& req, const std::string& client, int status, double ms) {
  if (g_opt.quiet) return;
  Value o = Value::object();
  o.set("client", Value::string(client));
  o.set("method", Value::string(req.method));
  o.set("path", Value::string(req.path));
  o.set("status", Value::number(status));
  o.set("latency_ms", Value::number(std::round(ms * 1000) / 1000));
  std::fprintf(stderr, "%s\n", barqjson::dump(o).c_str());
}

void serve_connection(int fd, std::string client) {
  struct Close {
    int fd;
    ~Close() {
      ::close(fd);
      --g_ctr.connections;
    }
  } closer{fd};
  timeval tv{};
  tv.tv_sec = 60;  // idle keep-alive connections are dropped after a minute
  setsockopt(fd, SOL_SOCKET, SO_RCVTIMEO, &tv, sizeof tv);
  int one = 1;
  setsockopt(fd, IPPROTO_TCP, TCP_NODELAY, &one, sizeof one);
  Conn conn(fd);
  for (;;) {
    Request req;
    const int rc = conn.read(req);
    if (rc < 0) return;
    if (rc > 0) {
      respond(fd, rc, "application/json", error_body(reason_phrase(rc), error_kind(rc)), false, "");
      return;
    }
    const double t0 = now_s();
    const std::string connection = lower(req.header("connection"));
    const bool keep = req.version == "HTTP/1.1" ? connection != "close" : connection == "keep-alive";
    const Outcome out = dispatch(fd, req, client, keep);
    if (req.path == "/v1/completions" || req.path == "/v1/chat/completions" || req.path == "/v1/responses") {
      if (out.status == 200) ++g_ctr.ok;
      else if (out.status >= 500) ++g_ctr.server_errors;
      else ++g_ctr.client_errors;
    }
    log_line(req, client, out.status, (now_s() - t0) * 1e3);
    if (out.close || !keep) return;
  }
}

int usage_error(const char* msg) {
  std::fprintf(stderr, "barq-http: %s\n", msg);
  std::fprintf(stderr,
               "usage: barq-http --socket PATH [--host ADDR] [--port N] [--model-id NAME] [--rpm N]\n"
               "                 [--max-conns N] [--engine-timeout S] [--drain-timeout S] [--api-key KEY] [--quiet]\n");
  return 2;
}

}  // namespace

int main(int argc, char** argv) {
  for (int i = 1; i < argc; ++i) {
    const std::string a = argv[i];
    auto val = [&](const char* name) -> const char* {
      if (i + 1 >= argc) {
        std::fprintf(stderr, "barq-http: %s needs a value\n", name);
        std::exit(2);
      }
      return argv[++i];
    };
    auto num = [&](const char* name, int lo) {
      const char* v = val(name);
      char* end = nullptr;
      const long x = std::strtol(v, &end, 10);
      if (*v == '\0' || *end != '\0' || x < lo || x > 1000000000L) {
        std::fprintf(stderr, "barq-http: bad value for %s: %s\n", name, v);
        std::exit(2);
      }
      return (int)x;
    };
    if (a == "--socket") g_opt.sockets.push_back(val("--socket"));
    else if (a == "--host") g_opt.host = val("--host");
    else if (a == "--port") g_opt.port = num("--port", 0);
    else if (a == "--model-id") g_opt.model_id = val("--model-id");
    else if (a == "--rpm") g_opt.rpm = num("--rpm", 0);
    else if (a == "--max-conns") g_opt.max_conns = num("--max-conns", 1);
    else if (a == "--engine-timeout") g_opt.engine_timeout_s = num("--engine-timeout", 1);
    else if (a == "--drain-timeout") g_opt.drain_s = num("--drain-timeout", 0);
    else if (a == "--api-key") g_opt.api_key = val("--api-key");
    else if (a == "--quiet") g_opt.quiet = true;
    else if (a == "-h" || a == "--help") {
      usage_error("OpenAI-compatible HTTP front end for a barq UDS server");
      return 0;
    }
    else return usage_error(("unknown argument " + a).c_str());
  }
  if (g_opt.port > 65535) return usage_error("port out of range");
  if (g_opt.sockets.empty()) g_opt.sockets.push_back("/tmp/barq-inference.sock");
  if (g_opt.api_key.empty())
    if (const char* k = std::getenv("BARQ_API_KEY")) g_opt.api_key = k;
  if ((int)g_opt.sockets.size() > EnginePool::kMax) return usage_error("too many --socket engines");
  signal(SIGPIPE, SIG_IGN);
  struct sigaction sa{};
  sa.sa_handler = on_stop_signal;
  sigaction(SIGTERM, &sa, nullptr);
  sigaction(SIGINT, &sa, nullptr);
  const int ls = ::socket(AF_INET, SOCK_STREAM, 0);
  if (ls < 0) return usage_error(std::strerror(errno));
  int one = 1;
  setsockopt(ls, SOL_SOCKET, SO_REUSEADDR, &one, sizeof one);
  sockaddr_in addr{};
  addr.sin_family = AF_INET;
  addr.sin_port = htons((uint16_t)g_opt.port);
  if (inet_pton(AF_INET, g_opt.host.c_str(), &addr.sin_addr) != 1) return usage_error("--host must be an IPv4 address");
  if (::bind(ls, reinterpret_cast<sockaddr*>(&addr), sizeof addr) != 0 || ::listen(ls, 512) != 0) {
    std::fprintf(stderr, "barq-http: cannot listen on %s:%d: %s\n", g_opt.host.c_str(), g_opt.port,
                 std::strerror(errno));
    return 2;
  }
  socklen_t len = sizeof addr;
  getsockname(ls, reinterpret_cast<sockaddr*>(&addr), &len);
  // the bound port (useful with --port 0) on stdout, flushed, for whoever started the process
  std::printf("barq-http listening on %s:%d (engine socket %s%s)\n", g_opt.host.c_str(), ntohs(addr.sin_port),
              g_opt.sockets[0].c_str(), g_opt.sockets.size() > 1 ? " and more" : "");
  std::fflush(stdout);
  while (!g_stop) {
    pollfd pl{ls, POLLIN, 0};
    if (::poll(&pl, 1, 200) <= 0) continue;  // wakes up to notice a stop signal
    sockaddr_in peer{};
    socklen_t plen = sizeof peer;
    const int fd = ::accept(ls, reinterpret_cast<sockaddr*>(&peer), &plen);
    if (fd < 0) {
      if (errno == EINTR || errno == ECONNABORTED || errno == EMFILE || errno == ENFILE || errno == EAGAIN) continue;
      std::fprintf(stderr, "barq-http: accept: %s\n", std::strerror(errno));
      return 1;
    }
    char host[INET_ADDRSTRLEN] = "unknown";
    inet_ntop(AF_INET, &peer.sin_addr, host, sizeof host);
    if (++g_ctr.connections > g_opt.max_conns) {
      respond(fd, 503, "application/json", error_body("too many connections", "overloaded_error"), false, "");
      ::close(fd);
      --g_ctr.connections;
      continue;
    }
    std::thread(serve_connection, fd, std::string(host)).detach();
  }
  // graceful stop: no new connections; generations in flight get up to --drain-timeout seconds
  ::close(ls);
  const double t0 = now_s();
  while (g_ctr.active > 0 && now_s() - t0 < g_opt.drain_s) usleep(50 * 1000);
  if (!g_opt.quiet)
    std::fprintf(stderr, "barq-http: stopped (%lld request(s) still in flight)\n", (long long)g_ctr.active.load());
  std::fflush(stdout);
  std::_Exit(0);  // detached connection threads end with the process
}
