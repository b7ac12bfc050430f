// Request ingest (host code): the client's path from socket bytes to the rows
// process_batch steps, and the response encoder (include/b2e.h).
//
// The reference decodes every newline-delimited line with json.loads into a
// dataclass (protocol.py:86-103), queues one PendingRequest object per request
// in a per-symbol queue.Queue (client.py:156-173), drains all queues at once
// (client.py:202-220) and builds rounds from Python float lists
// (example_model.py:885-899). Here a line that json.loads would turn into a
// well-typed InferenceRequest is parsed straight into per-symbol arrays of
// unique ids and float32 features; anything else (other message types, bad
// JSON, unusual field types) is handed back whole to the caller, whose decoder
// is the reference's own, so no line is ever read differently from it.
#include <algorithm>
#include <atomic>
#include <charconv>
#include <condition_variable>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <deque>
#include <functional>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

#include "../../include/b2e.h"
#include "common.cuh"

namespace b2e {
int abi_call(const std::function<void()>& f);
}  // namespace b2e

using namespace b2e;

namespace {

// ---- JSON over one line, accepting exactly what Python's json.loads accepts
// for the parts read natively (json/scanner.py, json/decoder.py): whitespace
// " \t\n\r"; strings with the escapes \" \\ \/ \b \f \n \r \t \uXXXX and no raw
// control characters; numbers matching -?(0|[1-9]\d*)(\.\d+)?([eE][-+]?\d+)?;
// NaN, Infinity and -Infinity. Bytes >= 0x80 are left to the caller's decoder
// (it checks UTF-8 first), as are lone surrogates.
struct Reader {
  const char* p;
  const char* e;

  void ws() {
    while (p < e && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) ++p;
  }
  bool lit(const char* s) {
    const size_t n = std::strlen(s);
    if (size_t(e - p) >= n && std::memcmp(p, s, n) == 0) {
      p += n;
      return true;
    }
    return false;
  }
  bool peek(char c) const { return p < e && *p == c; }

  static int hex4(const char* q) {
    int v = 0;
    for (int i = 0; i < 4; ++i) {
      const char c = q[i];
      int d;
      if (c >= '0' && c <= '9') d = c - '0';
      else if (c >= 'a' && c <= 'f') d = c - 'a' + 10;
      else if (c >= 'A' && c <= 'F') d = c - 'A' + 10;
      else return -1;
      v = v * 16 + d;
    }
    return v;
  }
  static void utf8(std::string* out, uint32_t cp) {
    if (cp < 0x80) {
      out->push_back(char(cp));
    } else if (cp < 0x800) {
      out->push_back(char(0xC0 | (cp >> 6)));
      out->push_back(char(0x80 | (cp & 0x3F)));
    } else if (cp < 0x10000) {
      out->push_back(char(0xE0 | (cp >> 12)));
      out->push_back(char(0x80 | ((cp >> 6) & 0x3F)));
      out->push_back(char(0x80 | (cp & 0x3F)));
    } else {
      out->push_back(char(0xF0 | (cp >> 18)));
      out->push_back(char(0x80 | ((cp >> 12) & 0x3F)));
      out->push_back(char(0x80 | ((cp >> 6) & 0x3F)));
      out->push_back(char(0x80 | (cp & 0x3F)));
    }
  }
  // At '"'. False: not a string this reader takes.
  bool string(std::string* out) {
    if (!peek('"')) return false;
    ++p;
    if (out) out->clear();
    while (p < e) {
      const unsigned char c = static_cast<unsigned char>(*p);
      if (c == '"') {
        ++p;
        return true;
      }
      if (c < 0x20 || c >= 0x80) return false;
      if (c != '\\') {
        if (out) out->push_back(char(c));
        ++p;
        continue;
      }
      if (e - p < 2) return false;
      const char x = p[1];
      p += 2;
      char lit_c = 0;
      switch (x) {
        case '"': lit_c = '"'; break;
        case '\\': lit_c = '\\'; break;
        case '/': lit_c = '/'; break;
        case 'b': lit_c = '\b'; break;
        case 'f': lit_c = '\f'; break;
        case 'n': lit_c = '\n'; break;
        case 'r': lit_c = '\r'; break;
        case 't': lit_c = '\t'; break;
        case 'u': {
          if (e - p < 4) return false;
          int cp = hex4(p);
          if (cp < 0) return false;
          p += 4;
          if (cp >= 0xDC00 && cp <= 0xDFFF) return false;  // lone low surrogate
          if (cp >= 0xD800 && cp <= 0xDBFF) {
            if (e - p < 6 || p[0] != '\\' || p[1] != 'u') return false;  // lone high surrogate
            const int lo = hex4(p + 2);
            if (lo < 0xDC00 || lo > 0xDFFF) return false;
            p += 6;
            cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
          }
          if (out) utf8(out, uint32_t(cp));
          continue;
        }
        default: return false;
      }
      if (out) out->push_back(lit_c);
    }
    return false;
  }
  // A number token, or NaN / Infinity / -Infinity. is_int: no fraction and no
  // exponent (json.loads makes it a Python int). digits: its digit count.
  bool number(double* v, bool* is_int, int* digits) {
    if (p < e && (*p == 'N' || *p == 'I' || (*p == '-' && p + 1 < e && p[1] == 'I'))) {
      *is_int = false;
      *digits = 0;
      if (lit("NaN")) *v = std::nan("");
      else if (lit("Infinity")) *v = HUGE_VAL;
      else if (lit("-Infinity")) *v = -HUGE_VAL;
      else return false;
      return true;
    }
    const char* s = p;
    const char* q = p;
    if (q < e && *q == '-') ++q;
    if (q >= e) return false;
    int nd = 0;
    if (*q == '0') {
      ++q;
      nd = 1;
    } else if (*q >= '1' && *q <= '9') {
      while (q < e && *q >= '0' && *q <= '9') ++q, ++nd;
    } else {
      return false;
    }
    bool integral = true;
    if (q + 1 < e && *q == '.' && q[1] >= '0' && q[1] <= '9') {
      integral = false;
      ++q;
      while (q < e && *q >= '0' && *q <= '9') ++q;
    }
    if (q < e && (*q == 'e' || *q == 'E')) {
      const char* r = q + 1;
      if (r < e && (*r == '+' || *r == '-')) ++r;
      if (r < e && *r >= '0' && *r <= '9') {
        integral = false;
        while (r < e && *r >= '0' && *r <= '9') ++r;
        q = r;
      }
    }
    const auto res = std::from_chars(s, q, *v);  // correctly rounded, like float(str)
    if (res.ec == std::errc::result_out_of_range) {
      // beyond the finite doubles (or below the smallest): strtod rounds these
      // to +-inf, a subnormal or +-0 as float(str) does (in the C numeric
      // locale, which a Python process keeps unless it sets LC_NUMERIC)
      const std::string tok(s, size_t(q - s));
      *v = std::strtod(tok.c_str(), nullptr);
    } else if (res.ec != std::errc() || res.ptr != q) {
      return false;
    }
    p = q;
    *is_int = integral;
    *digits = nd;
    return true;
  }
  // Any value (depth-limited like the reference's recursion limit would be).
  bool skip(int depth) {
    if (depth > 256) return false;
    ws();
    if (p >= e) return false;
    if (*p == '"') return string(nullptr);
    if (*p == '{') {
      ++p;
      ws();
      if (peek('}')) {
        ++p;
        return true;
      }
      for (;;) {
        ws();
        if (!string(nullptr)) return false;
        ws();
        if (!peek(':')) return false;
        ++p;
        if (!skip(depth + 1)) return false;
        ws();
        if (peek(',')) {
          ++p;
          continue;
        }
        if (peek('}')) {
          ++p;
          return true;
        }
        return false;
      }
    }
    if (*p == '[') {
      ++p;
      ws();
      if (peek(']')) {
        ++p;
        return true;
      }
      for (;;) {
        if (!skip(depth + 1)) return false;
        ws();
        if (peek(',')) {
          ++p;
          continue;
        }
        if (peek(']')) {
          ++p;
          return true;
        }
        return false;
      }
    }
    if (lit("true") || lit("false") || lit("null")) return true;
    double v;
    bool ii;
    int nd;
    return number(&v, &ii, &nd);
  }
};

// One decoded InferenceRequest (protocol.py:28-34).
struct Request {
  std::vector<int64_t> uids;
  std::vector<std::string> symbols;
  std::vector<float> feats;      // rows of F, for every well-formed row
  std::vector<uint8_t> row_ok;   // row r has F numbers json.loads maps to the same float32 here
  size_t rows = 0;
};

enum class Field { kNone, kType, kUids, kSymbols, kFeatures, kTimestamp };

// The line as json.loads + ProtocolHandler.decode would see it. True: an
// inference_request this code reads natively into `q`.
bool parse_request(const char* s, size_t n, int F, Request* q, std::string* mtype) {
  Reader r{s, s + n};
  r.ws();
  if (!r.peek('{')) return false;
  ++r.p;
  bool have_type = false, have_u = false, have_s = false, have_f = false, have_t = false;
  bool u_ok = false, s_ok = false, f_ok = false;
  std::string key;
  r.ws();
  if (r.peek('}')) return false;  // no message_type
  for (;;) {
    r.ws();
    if (!r.string(&key)) return false;
    r.ws();
    if (!r.peek(':')) return false;
    ++r.p;
    r.ws();
    Field f = Field::kNone;
    if (key == "message_type") f = Field::kType;
    else if (key == "unique_ids") f = Field::kUids;
    else if (key == "symbols") f = Field::kSymbols;
    else if (key == "features") f = Field::kFeatures;
    else if (key == "timestamp") f = Field::kTimestamp;
    if (f == Field::kNone) return false;  // InferenceRequest(**d) would reject the key
    if (f == Field::kType) {
      have_type = true;
      if (!r.peek('"')) {
        if (!r.skip(0)) return false;
        mtype->assign("\x01");  // not a string: never a known type
      } else if (!r.string(mtype)) {
        return false;
      }
    } else if (f == Field::kTimestamp) {
      have_t = true;  // any value: InferenceRequest does not check it
      if (!r.skip(0)) return false;
    } else if (f == Field::kUids) {
      have_u = true;
      u_ok = false;
      q->uids.clear();
      if (!r.peek('[')) {
        if (!r.skip(0)) return false;
      } else {
        ++r.p;
        r.ws();
        bool good = true;
        if (r.peek(']')) {
          ++r.p;
        } else {
          for (;;) {
            r.ws();
            const char* t0 = r.p;
            double v;
            bool ii;
            int nd;
            if (r.peek('-') || (r.p < r.e && *r.p >= '0' && *r.p <= '9') || r.peek('N') || r.peek('I')) {
              if (!r.number(&v, &ii, &nd)) return false;
              int64_t u = 0;
              if (ii && std::from_chars(t0, r.p, u).ec == std::errc()) q->uids.push_back(u);
              else good = false;  // float id, or beyond int64
            } else {
              if (!r.skip(0)) return false;
              good = false;
            }
            r.ws();
            if (r.peek(',')) {
              ++r.p;
              continue;
            }
            if (r.peek(']')) {
              ++r.p;
              break;
            }
            return false;
          }
        }
        u_ok = good;
      }
    } else if (f == Field::kSymbols) {
      have_s = true;
      s_ok = false;
      q->symbols.clear();
      if (!r.peek('[')) {
        if (!r.skip(0)) return false;
      } else {
        ++r.p;
        r.ws();
        bool good = true;
        if (r.peek(']')) {
          ++r.p;
        } else {
          std::string sym;
          for (;;) {
            r.ws();
            if (r.peek('"')) {
              if (!r.string(&sym)) return false;
              q->symbols.push_back(sym);
            } else {
              if (!r.skip(0)) return false;
              good = false;
            }
            r.ws();
            if (r.peek(',')) {
              ++r.p;
              continue;
            }
            if (r.peek(']')) {
              ++r.p;
              break;
            }
            return false;
          }
        }
        s_ok = good;
      }
    } else {  // features
      have_f = true;
      f_ok = false;
      q->feats.clear();
      q->row_ok.clear();
      q->rows = 0;
      if (!r.peek('[')) {
        if (!r.skip(0)) return false;
      } else {
        ++r.p;
        r.ws();
        bool good = true;
        if (r.peek(']')) {
          ++r.p;
        } else {
          for (;;) {
            r.ws();
            if (!r.peek('[')) {
              if (!r.skip(0)) return false;
              q->feats.resize(q->feats.size() + size_t(F), 0.f);
              q->row_ok.push_back(0);
            } else {
              ++r.p;
              r.ws();
              const size_t base = q->feats.size();
              q->feats.resize(base + size_t(F), 0.f);
              int k = 0;
              bool row_good = true;
              if (r.peek(']')) {
                ++r.p;
              } else {
                for (;;) {
                  r.ws();
                  double v;
                  bool ii;
                  int nd;
                  const char c = r.p < r.e ? *r.p : 0;
                  if (c == '-' || (c >= '0' && c <= '9') || c == 'N' || c == 'I') {
                    if (!r.number(&v, &ii, &nd)) return false;
                    // a long Python int may round differently on its way to float32
                    if (ii && nd > 15) row_good = false;
                    if (ii && v == 0.0) v = 0.0;  // int("-0") is 0: no negative zero
                    if (k < F) q->feats[base + size_t(k)] = static_cast<float>(v);
                  } else {
                    if (!r.skip(0)) return false;
                    row_good = false;
                  }
                  ++k;
                  r.ws();
                  if (r.peek(',')) {
                    ++r.p;
                    continue;
                  }
                  if (r.peek(']')) {
                    ++r.p;
                    break;
                  }
                  return false;
                }
              }
              q->row_ok.push_back(row_good && k == F);
            }
            ++q->rows;
            r.ws();
            if (r.peek(',')) {
              ++r.p;
              continue;
            }
            if (r.peek(']')) {
              ++r.p;
              break;
            }
            return false;
          }
        }
        f_ok = good;
      }
    }
    r.ws();
    if (r.peek(',')) {
      ++r.p;
      continue;
    }
    if (r.peek('}')) {
      ++r.p;
      break;
    }
    return false;
  }
  r.ws();
  if (r.p != r.e) return false;  // trailing bytes: json.loads raises
  if (!have_type || *mtype != "inference_request") return false;
  if (!(have_u && have_s && have_f && have_t) || !(u_ok && s_ok && f_ok)) return false;
  const size_t m = std::min({q->uids.size(), q->symbols.size(), q->rows});
  for (size_t i = 0; i < m; ++i)
    if (!q->row_ok[i]) return false;
  return true;
}

// float.__repr__ as json.dumps writes it (Objects/floatobject.c float_repr:
// the shortest digits that round-trip, fixed notation for decimal exponents
// -4 < decpt <= 16 with ".0" added to whole numbers, else d.ddde+XX);
// NaN / Infinity / -Infinity for the non-finite values (json allow_nan).
void py_float(std::string* out, double x) {
  if (std::isnan(x)) {
    out->append("NaN");
    return;
  }
  if (std::isinf(x)) {
    out->append(x > 0 ? "Infinity" : "-Infinity");
    return;
  }
  if (x == 0.0) {
    out->append(std::signbit(x) ? "-0.0" : "0.0");
    return;
  }
  char buf[64];
  const auto res = std::to_chars(buf, buf + sizeof(buf), x, std::chars_format::scientific);
  const char* q = buf;
  if (*q == '-') {
    out->push_back('-');
    ++q;
  }
  char digits[32];
  int nd = 0;
  const char* t = q;
  for (; t < res.ptr && *t != 'e'; ++t)
    if (*t != '.') digits[nd++] = *t;
  int e10 = 0;
  std::from_chars(t + 1 + (t[1] == '+' ? 1 : 0), res.ptr, e10);
  const int decpt = e10 + 1;
  if (decpt <= -4 || decpt > 16) {
    out->push_back(digits[0]);
    if (nd > 1) {
      out->push_back('.');
      out->append(digits + 1, size_t(nd - 1));
    }
    out->push_back('e');
    const int ae = e10 < 0 ? -e10 : e10;
    out->push_back(e10 < 0 ? '-' : '+');
    if (ae < 10) out->push_back('0');
    out->append(std::to_string(ae));
  } else if (decpt <= 0) {
    out->append("0.");
    out->append(size_t(-decpt), '0');
    out->append(digits, size_t(nd));
  } else if (decpt >= nd) {
    out->append(digits, size_t(nd));
    out->append(size_t(decpt - nd), '0');
    out->append(".0");
  } else {
    out->append(digits, size_t(decpt));
    out->push_back('.');
    out->append(digits + decpt, size_t(nd - decpt));
  }
}

// A fixed set of worker threads that run job(i) for i in [0, n) together with
// the calling thread; run() returns when every job is done.
class Pool {
 public:
  explicit Pool(int threads) {
    for (int t = 0; t < threads; ++t) th_.emplace_back([this] { loop(); });
  }
  ~Pool() {
    {
      std::lock_guard<std::mutex> lk(m_);
      stop_ = true;
    }
    cv_.notify_all();
    for (auto& t : th_) t.join();
  }
  int threads() const { return int(th_.size()) + 1; }
  void run(int n, const std::function<void(int)>& job) {
    {
      std::lock_guard<std::mutex> lk(m_);
      job_ = &job;
      n_ = n;
      next_.store(0);
      pending_ = int(th_.size());
      ++gen_;
    }
    cv_.notify_all();
    work();
    std::unique_lock<std::mutex> lk(m_);
    done_.wait(lk, [&] { return pending_ == 0; });
    job_ = nullptr;
  }

 private:
  void work() {
    for (int i; (i = next_.fetch_add(1)) < n_;) (*job_)(i);
  }
  void loop() {
    uint64_t seen = 0;
    for (;;) {
      std::unique_lock<std::mutex> lk(m_);
      cv_.wait(lk, [&] { return stop_ || gen_ != seen; });
      if (stop_) return;
      seen = gen_;
      lk.unlock();
      work();
      lk.lock();
      if (--pending_ == 0) done_.notify_all();
    }
  }
  std::vector<std::thread> th_;
  std::mutex m_;
  std::condition_variable cv_, done_;
  const std::function<void(int)>* job_ = nullptr;
  int n_ = 0, pending_ = 0;
  std::atomic<int> next_{0};
  uint64_t gen_ = 0;
  bool stop_ = false;
};

}  // namespace

struct b2e_ingest {
  // Every entry point holds this while it touches the handle: a receive thread
  // may feed (and so grow `syms`) while a process thread takes or names symbols.
  mutable std::mutex mu;
  struct Sym {
    std::string name;
    std::vector<int64_t> uids;  // queued requests, oldest first, from `head`
    std::vector<float> feats;
    std::vector<uint64_t> seqs;  // arrival order of each queued request
    size_t head = 0;             // requests before it were taken by take_batch
    size_t len() const { return uids.size() - head; }
    void clear() {
      uids.clear();
      feats.clear();
      seqs.clear();
      head = 0;
    }
  };
  int F = 0;
  int max_queue = 0;  // <= 0: unbounded, like queue.Queue(maxsize=0)
  std::string buf;    // bytes not yet split into lines, from `off`
  size_t off = 0;
  std::vector<Sym> syms;
  std::unordered_map<std::string, int32_t> ids;
  std::vector<int32_t> active;  // symbols with queued requests
  uint64_t seq = 0;             // arrivals so far
  std::deque<std::string> others;
  std::deque<int32_t> drops;
  int64_t queued = 0;
  Request req;
  std::string mtype;
  // lines parsed side by side, then queued in order
  std::unique_ptr<Pool> pool;
  struct Parsed {
    Request req;
    std::string mtype;
    bool ok = false;
  };
  std::vector<Parsed> parsed;
  std::vector<std::pair<size_t, size_t>> spans;  // (offset in buf, length) of complete lines

  int32_t id_of(const std::string& s) {
    auto it = ids.find(s);
    if (it != ids.end()) return it->second;
    const int32_t id = int32_t(syms.size());
    syms.push_back(Sym{s, {}, {}, {}, 0});
    ids.emplace(s, id);
    return id;
  }
  // _handle_request for one request (client.py:162-173).
  bool push(int32_t id, int64_t uid, const float* f) {
    Sym& y = syms[size_t(id)];
    if (max_queue > 0 && y.len() >= size_t(max_queue)) {
      drops.push_back(id);
      return false;
    }
    if (y.len() == 0) active.push_back(id);
    y.uids.push_back(uid);
    y.feats.insert(y.feats.end(), f, f + F);
    y.seqs.push_back(seq++);
    ++queued;
    return true;
  }
  // One complete line (no newline), parsed (`ok`: a request line in `q`):
  // queue its requests (true) or keep it whole.
  bool line(const char* s, size_t n, bool ok, const Request& q, int32_t* n_req, int32_t* n_other) {
    if (n == 0) return true;  // SocketReader skips empty lines
    if (!ok) {
      others.emplace_back(s, n);
      ++*n_other;
      return false;
    }
    const size_t m = std::min({q.uids.size(), q.symbols.size(), q.rows});
    for (size_t i = 0; i < m; ++i)
      if (push(id_of(q.symbols[i]), q.uids[i], q.feats.data() + i * size_t(F))) ++*n_req;
    return true;
  }
};

namespace {
b2e_ingest& G(b2e_ingest* g) {
  B2E_CHECK(g != nullptr, kErrInvalid, "null ingest handle");
  return *g;
}
const b2e_ingest& G(const b2e_ingest* g) {
  B2E_CHECK(g != nullptr, kErrInvalid, "null ingest handle");
  return *g;
}
void give(const std::string& s, char* buf, int64_t cap, int64_t* len, bool* taken) {
  *len = int64_t(s.size());
  *taken = false;
  if (int64_t(s.size()) > cap) return;
  B2E_CHECK(buf != nullptr || s.empty(), kErrInvalid, "null output buffer");
  if (!s.empty()) std::memcpy(buf, s.data(), s.size());
  *taken = true;
}
}  // namespace

extern "C" {

int b2e_ingest_create(int32_t num_features, int32_t max_queue, b2e_ingest** out) {
  return abi_call([&] {
    B2E_CHECK(out != nullptr, kErrInvalid, "null output handle");
    *out = nullptr;
    B2E_CHECK(num_features > 0 && num_features <= 65536, kErrInvalid, "num_features must be in 1..65536");
    auto* g = new b2e_ingest;
    g->F = num_features;
    g->max_queue = max_queue;
    const unsigned hw = std::thread::hardware_concurrency();
    const int threads = int(std::min(8u, hw > 0 ? hw : 1u));
    if (threads > 1) g->pool = std::make_unique<Pool>(threads - 1);
    *out = g;
  });
}

void b2e_ingest_destroy(b2e_ingest* g) { delete g; }

int b2e_ingest_set_threads(b2e_ingest* g, int32_t threads) {
  return abi_call([&] {
    b2e_ingest& s = G(g);
    std::lock_guard<std::mutex> lk(s.mu);
    B2E_CHECK(threads >= 1 && threads <= 256, kErrInvalid, "threads must be in 1..256");
    s.pool.reset();
    if (threads > 1) s.pool = std::make_unique<Pool>(threads - 1);
  });
}

int b2e_ingest_feed(b2e_ingest* g, const char* data, int64_t len, int32_t* n_requests, int32_t* n_other) {
  return abi_call([&] {
    b2e_ingest& s = G(g);
    std::lock_guard<std::mutex> lk(s.mu);
    B2E_CHECK(len >= 0 && (len == 0 || data != nullptr), kErrInvalid, "bad byte range");
    if (len > 0) s.buf.append(data, size_t(len));
    int32_t nr = 0, no = 0;
    // the complete lines from `off`
    s.spans.clear();
    size_t bytes = 0;
    for (size_t o = s.off; o < s.buf.size();) {
      const char* p = s.buf.data() + o;
      const char* nl = static_cast<const char*>(std::memchr(p, '\n', s.buf.size() - o));
      if (!nl) break;
      s.spans.emplace_back(o, size_t(nl - p));
      bytes += size_t(nl - p);
      o += size_t(nl - p) + 1;
    }
    const int nl = int(s.spans.size());
    if (s.pool && nl > 1 && bytes >= (size_t(64) << 10)) {
      // parse side by side; the queue order below is the line order
      if (s.parsed.size() < size_t(nl)) s.parsed.resize(size_t(nl));
      const std::function<void(int)> job = [&](int i) {
        b2e_ingest::Parsed& q = s.parsed[size_t(i)];
        q.ok = s.spans[size_t(i)].second > 0 &&
               parse_request(s.buf.data() + s.spans[size_t(i)].first, s.spans[size_t(i)].second, s.F, &q.req, &q.mtype);
      };
      s.pool->run(nl, job);
      for (int i = 0; i < nl; ++i) {
        const auto sp = s.spans[size_t(i)];
        s.off = sp.first + sp.second + 1;
        if (!s.line(s.buf.data() + sp.first, sp.second, s.parsed[size_t(i)].ok, s.parsed[size_t(i)].req, &nr, &no))
          break;  // the caller reads this line first; the lines after it are parsed again next time
      }
    } else {
      for (int i = 0; i < nl; ++i) {
        const auto sp = s.spans[size_t(i)];
        s.off = sp.first + sp.second + 1;
        const bool ok = sp.second > 0 && parse_request(s.buf.data() + sp.first, sp.second, s.F, &s.req, &s.mtype);
        if (!s.line(s.buf.data() + sp.first, sp.second, ok, s.req, &nr, &no)) break;
      }
    }
    if (s.off == s.buf.size() || s.off > (size_t(1) << 20)) {
      s.buf.erase(0, s.off);
      s.off = 0;
    }
    if (n_requests) *n_requests = nr;
    if (n_other) *n_other = no;
  });
}

int b2e_ingest_next_other(b2e_ingest* g, char* buf, int64_t cap, int64_t* len) {
  return abi_call([&] {
    b2e_ingest& s = G(g);
    std::lock_guard<std::mutex> lk(s.mu);
    B2E_CHECK(len != nullptr, kErrInvalid, "null length");
    if (s.others.empty()) {
      *len = -1;
      return;
    }
    bool taken = false;
    give(s.others.front(), buf, cap, len, &taken);
    if (taken) s.others.pop_front();
  });
}

int b2e_ingest_push(b2e_ingest* g, int64_t unique_id, const char* symbol, int64_t symbol_len, const float* features,
                    int32_t* queued) {
  return abi_call([&] {
    b2e_ingest& s = G(g);
    std::lock_guard<std::mutex> lk(s.mu);
    B2E_CHECK(symbol_len >= 0 && (symbol_len == 0 || symbol != nullptr), kErrInvalid, "bad symbol bytes");
    B2E_CHECK(features != nullptr, kErrInvalid, "null features");
    const bool ok = s.push(s.id_of(std::string(symbol ? symbol : "", size_t(symbol_len))), unique_id, features);
    if (queued) *queued = ok ? 1 : 0;
  });
}

int b2e_ingest_next_drop(b2e_ingest* g, int32_t* symbol) {
  return abi_call([&] {
    b2e_ingest& s = G(g);
    std::lock_guard<std::mutex> lk(s.mu);
    B2E_CHECK(symbol != nullptr, kErrInvalid, "null output");
    if (s.drops.empty()) {
      *symbol = -1;
      return;
    }
    *symbol = s.drops.front();
    s.drops.pop_front();
  });
}

int b2e_ingest_pending(const b2e_ingest* g, int64_t* rows) {
  return abi_call([&] {
    B2E_CHECK(rows != nullptr, kErrInvalid, "null output");
    const b2e_ingest& s = G(g);
    std::lock_guard<std::mutex> lk(s.mu);
    *rows = s.queued;
  });
}

int b2e_ingest_symbol_count(const b2e_ingest* g, int32_t* n) {
  return abi_call([&] {
    B2E_CHECK(n != nullptr, kErrInvalid, "null output");
    const b2e_ingest& s = G(g);
    std::lock_guard<std::mutex> lk(s.mu);
    *n = int32_t(s.syms.size());
  });
}

int b2e_ingest_symbol_name(const b2e_ingest* g, int32_t symbol, char* buf, int64_t cap, int64_t* len) {
  return abi_call([&] {
    const b2e_ingest& s = G(g);
    std::lock_guard<std::mutex> lk(s.mu);
    B2E_CHECK(len != nullptr, kErrInvalid, "null length");
    B2E_CHECK(symbol >= 0 && size_t(symbol) < s.syms.size(), kErrInvalid, "unknown symbol id");
    bool taken = false;
    give(s.syms[size_t(symbol)].name, buf, cap, len, &taken);
  });
}

int b2e_ingest_take(b2e_ingest* g, int64_t cap, int32_t* symbols, int64_t* unique_ids, float* features,
                    int32_t* round_rows, int32_t* n_rounds, int64_t* n_rows) {
  return abi_call([&] {
    b2e_ingest& s = G(g);
    std::lock_guard<std::mutex> lk(s.mu);
    B2E_CHECK(n_rounds && n_rows, kErrInvalid, "null output");
    B2E_CHECK(cap >= s.queued, kErrInvalid, "take: buffers hold fewer rows than are pending");
    B2E_CHECK(s.queued == 0 || (symbols && unique_ids && features && round_rows), kErrInvalid, "null output buffer");
    std::sort(s.active.begin(), s.active.end());  // ids are first-sight order: the dict order
    size_t depth = 0;
    for (int32_t id : s.active) depth = std::max(depth, s.syms[size_t(id)].len());
    const size_t F = size_t(s.F);
    int64_t row = 0;
    int32_t rounds = 0;
    std::vector<int32_t> live = s.active;
    for (size_t k = 0; k < depth; ++k) {
      int32_t in_round = 0;
      size_t w = 0;
      for (int32_t id : live) {
        const b2e_ingest::Sym& y = s.syms[size_t(id)];
        if (y.len() <= k) continue;
        live[w++] = id;
        symbols[row] = id;
        unique_ids[row] = y.uids[y.head + k];
        std::memcpy(features + size_t(row) * F, y.feats.data() + (y.head + k) * F, F * sizeof(float));
        ++row;
        ++in_round;
      }
      live.resize(w);
      round_rows[rounds++] = in_round;
    }
    for (int32_t id : s.active) s.syms[size_t(id)].clear();
    s.active.clear();
    s.queued = 0;
    *n_rounds = rounds;
    *n_rows = row;
  });
}

int b2e_ingest_take_batch(b2e_ingest* g, int32_t max_rows, int32_t* symbols, int64_t* unique_ids, float* features,
                          int32_t* n_rows) {
  return abi_call([&] {
    b2e_ingest& s = G(g);
    std::lock_guard<std::mutex> lk(s.mu);
    B2E_CHECK(n_rows != nullptr && max_rows >= 0, kErrInvalid, "bad output");
    const size_t n = std::min(size_t(max_rows), s.active.size());
    B2E_CHECK(n == 0 || (symbols && unique_ids && features), kErrInvalid, "null output buffer");
    // the n symbols whose oldest queued request arrived first, in that order
    std::vector<std::pair<uint64_t, int32_t>> heads;
    heads.reserve(s.active.size());
    for (int32_t id : s.active) {
      const b2e_ingest::Sym& y = s.syms[size_t(id)];
      heads.emplace_back(y.seqs[y.head], id);
    }
    std::partial_sort(heads.begin(), heads.begin() + std::ptrdiff_t(n), heads.end());
    const size_t F = size_t(s.F);
    bool emptied = false;
    for (size_t r = 0; r < n; ++r) {
      b2e_ingest::Sym& y = s.syms[size_t(heads[r].second)];
      symbols[r] = heads[r].second;
      unique_ids[r] = y.uids[y.head];
      std::memcpy(features + r * F, y.feats.data() + y.head * F, F * sizeof(float));
      ++y.head;
      if (y.len() == 0) {
        y.clear();
        emptied = true;
      } else if (y.head >= 64 && 2 * y.head >= y.uids.size()) {  // keep a long-lived queue compact
        y.uids.erase(y.uids.begin(), y.uids.begin() + std::ptrdiff_t(y.head));
        y.seqs.erase(y.seqs.begin(), y.seqs.begin() + std::ptrdiff_t(y.head));
        y.feats.erase(y.feats.begin(), y.feats.begin() + std::ptrdiff_t(y.head * F));
        y.head = 0;
      }
    }
    if (emptied) {
      size_t w = 0;
      for (int32_t id : s.active)
        if (s.syms[size_t(id)].len() > 0) s.active[w++] = id;
      s.active.resize(w);
    }
    s.queued -= int64_t(n);
    *n_rows = int32_t(n);
  });
}

int b2e_encode_response(const int64_t* unique_ids, const float* predictions, int64_t n, int32_t n_out,
                        double client_timestamp, char* buf, int64_t cap, int64_t* len) {
  return abi_call([&] {
    B2E_CHECK(len != nullptr, kErrInvalid, "null length");
    B2E_CHECK(n >= 0 && n_out >= 0, kErrInvalid, "negative size");
    B2E_CHECK(n == 0 || (unique_ids && (n_out == 0 || predictions)), kErrInvalid, "null input");
    std::string o;
    o.reserve(size_t(n) * (24 + size_t(n_out) * 24) + 128);
    char ib[24];
    o.append("{\"unique_ids\": [");
    for (int64_t i = 0; i < n; ++i) {
      if (i) o.append(", ");
      const auto r = std::to_chars(ib, ib + sizeof(ib), unique_ids[i]);
      o.append(ib, size_t(r.ptr - ib));
    }
    o.append("], \"predictions\": [");
    for (int64_t i = 0; i < n; ++i) {
      if (i) o.append(", ");
      o.push_back('[');
      for (int32_t j = 0; j < n_out; ++j) {
        if (j) o.append(", ");
        py_float(&o, double(predictions[size_t(i) * size_t(n_out) + size_t(j)]));
      }
      o.push_back(']');
    }
    o.append("], \"client_timestamp\": ");
    py_float(&o, client_timestamp);
    o.append(", \"message_type\": \"inference_response\"}\n");
    bool taken = false;
    give(o, buf, cap, len, &taken);
  });
}

}  // extern "C"
