// The `.tune` version 2 store: checksummed canonical JSON lines behind the C ABI.
//
// Follows the reference autotuner's persistent cache (projects/titan-autotune/src/lib.rs:46-82:
// `Autotuner::open` on a `.tune` path, exact-key `get`/`insert`, `flush` writing a
// `# titan.tune version=2` header, sorted rows, a `.tune.tmp` file and a rename) with
// the persistence rules of docs/architecture/autotune-v2.md:9 that the Rust code
// leaves out: canonical JSONL, a checksum per record, an exclusive lock, merge with the
// records on disk, fsync of the temporary file, atomic rename, fsync of the directory.
//
// File format. Line 1 is `# titan.tune version=2`; every other line is the canonical
// JSON of {"checksum": C, "entry": E, "key": K} where K and E are JSON objects and C is
// the lowercase hex SHA-256 of the canonical {"entry": E, "key": K}. Canonical JSON is
// byte-identical to Python's json.dumps(obj, sort_keys=True, separators=(",", ":")):
// object members sorted by code point, no whitespace, ASCII only (\uXXXX escapes with
// lowercase hex, surrogate pairs above the BMP), integers as written ("-0" as "0"),
// floats in Python's shortest repr, NaN/Infinity/-Infinity as bare words. Files from
// the Python host and from this library are therefore interchangeable.
//
// Reading. The file is split into lines as Python's str.splitlines does; a file that
// is not valid UTF-8 contributes nothing (as a strict UTF-8 read would), a file whose
// first line is not the header contributes nothing and counts all its lines as
// ignored, blank lines are skipped, and a line that is not JSON, is not an object, lacks
// an object `key` or `entry`, or carries a wrong checksum is counted as ignored. Later
// lines win over earlier ones with the same key. The store keeps records as canonical
// strings and does not interpret the fields of a key or an entry.
#include <fcntl.h>
#include <sys/file.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <charconv>
#include <cmath>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "internal.hpp"
#include "json.hpp"

namespace {

using namespace tb::json;

const char kHeader[] = "# titan.tune version=2";

// ---------------------------------------------------------------- SHA-256 (FIPS 180-4)

// floor(v^(1/3)) and floor(v^(1/2)) of 128-bit integers by bisection.
uint64_t icbrt(unsigned __int128 v) {
  uint64_t lo = 0, hi = 1ull << 42;  // (2^42)^3 = 2^126 > every argument used here
  while (hi - lo > 1) {
    uint64_t mid = lo + (hi - lo) / 2;
    unsigned __int128 m = mid;
    if (m * m * m <= v) lo = mid; else hi = mid;
  }
  return lo;
}

uint64_t isqrt(unsigned __int128 v) {
  uint64_t lo = 0, hi = 1ull << 40;
  while (hi - lo > 1) {
    uint64_t mid = lo + (hi - lo) / 2;
    unsigned __int128 m = mid;
    if (m * m <= v) lo = mid; else hi = mid;
  }
  return lo;
}

// FIPS 180-4 §4.2.2 / §5.3.3: the round constants are the first 32 bits of the
// fractional parts of the cube roots of the first 64 primes, the initial hash the same
// of the square roots of the first 8. floor(cbrt(p) * 2^32) = floor(cbrt(p * 2^96)),
// whose low 32 bits are the fractional bits; the same holds for square roots with 2^64.
struct Sha256Constants {
  uint32_t k[64];
  uint32_t h0[8];
  Sha256Constants() {
    int n = 0;
    for (uint32_t p = 2; n < 64; ++p) {
      bool prime = true;
      for (uint32_t d = 2; d * d <= p; ++d)
        if (p % d == 0) { prime = false; break; }
      if (!prime) continue;
      k[n] = (uint32_t)icbrt((unsigned __int128)p << 96);
      if (n < 8) h0[n] = (uint32_t)isqrt((unsigned __int128)p << 64);
      ++n;
    }
  }
};

const Sha256Constants& sha_constants() {
  static const Sha256Constants c;
  return c;
}

inline uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }

void sha256_block(uint32_t h[8], const uint8_t* p, const uint32_t* k) {
  uint32_t w[64];
  for (int t = 0; t < 16; ++t)
    w[t] = (uint32_t)p[4 * t] << 24 | (uint32_t)p[4 * t + 1] << 16 | (uint32_t)p[4 * t + 2] << 8 | p[4 * t + 3];
  for (int t = 16; t < 64; ++t) {
    uint32_t s0 = rotr(w[t - 15], 7) ^ rotr(w[t - 15], 18) ^ (w[t - 15] >> 3);
    uint32_t s1 = rotr(w[t - 2], 17) ^ rotr(w[t - 2], 19) ^ (w[t - 2] >> 10);
    w[t] = w[t - 16] + s0 + w[t - 7] + s1;
  }
  uint32_t a = h[0], b = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], hh = h[7];
  for (int t = 0; t < 64; ++t) {
    uint32_t t1 = hh + (rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25)) + ((e & f) ^ (~e & g)) + k[t] + w[t];
    uint32_t t2 = (rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22)) + ((a & b) ^ (a & c) ^ (b & c));
    hh = g; g = f; f = e; e = d + t1; d = c; c = b; b = a; a = t1 + t2;
  }
  h[0] += a; h[1] += b; h[2] += c; h[3] += d; h[4] += e; h[5] += f; h[6] += g; h[7] += hh;
}

std::string sha256_hex(const uint8_t* data, size_t len) {
  const Sha256Constants& c = sha_constants();
  uint32_t h[8];
  std::copy(c.h0, c.h0 + 8, h);
  size_t full = len / 64;
  for (size_t i = 0; i < full; ++i) sha256_block(h, data + 64 * i, c.k);
  // Padding: 0x80, zeros to 56 mod 64, then the message length in bits, big-endian.
  uint8_t tail[128] = {};
  size_t rem = len - 64 * full;
  std::copy(data + 64 * full, data + len, tail);
  tail[rem] = 0x80;
  size_t tail_len = rem < 56 ? 64 : 128;
  uint64_t bits = (uint64_t)len * 8;
  for (int i = 0; i < 8; ++i) tail[tail_len - 1 - i] = (uint8_t)(bits >> (8 * i));
  for (size_t off = 0; off < tail_len; off += 64) sha256_block(h, tail + off, c.k);
  static const char hex[] = "0123456789abcdef";
  std::string out(64, '0');
  for (int i = 0; i < 8; ++i)
    for (int j = 0; j < 8; ++j) out[8 * i + j] = hex[(h[i] >> (28 - 4 * j)) & 15];
  return out;
}

// Python's str.isspace() set, used by str.strip().
bool py_space(uint32_t c) {
  return (c >= 0x09 && c <= 0x0D) || (c >= 0x1C && c <= 0x20) || c == 0x85 || c == 0xA0 || c == 0x1680 ||
         (c >= 0x2000 && c <= 0x200A) || c == 0x2028 || c == 0x2029 || c == 0x202F || c == 0x205F || c == 0x3000;
}

// str.strip() of valid UTF-8.
std::string py_strip(const std::string& s) {
  std::vector<std::pair<size_t, uint32_t>> cps;  // (byte offset, code point)
  const uint8_t* base = (const uint8_t*)s.data();
  const uint8_t* p = base;
  const uint8_t* end = base + s.size();
  while (p < end) {
    size_t off = (size_t)(p - base);
    cps.emplace_back(off, decode_cp(p));
  }
  size_t b = 0, e = cps.size();
  while (b < e && py_space(cps[b].second)) ++b;
  while (e > b && py_space(cps[e - 1].second)) --e;
  if (b == e) return std::string();
  size_t from = cps[b].first;
  size_t to = e < cps.size() ? cps[e].first : s.size();
  return s.substr(from, to - from);
}

// str.splitlines() of valid UTF-8: breaks at \n, \r, \r\n, \v, \f, \x1c, \x1d, \x1e,
// U+0085, U+2028 and U+2029; no empty line after a final break.
std::vector<std::string> py_splitlines(const std::string& s) {
  std::vector<std::string> lines;
  size_t start = 0, i = 0, n = s.size();
  const uint8_t* u = (const uint8_t*)s.data();
  while (i < n) {
    size_t brk = 0;
    uint8_t b = u[i];
    if (b == '\r') brk = (i + 1 < n && u[i + 1] == '\n') ? 2 : 1;
    else if (b == '\n' || b == 0x0B || b == 0x0C || b == 0x1C || b == 0x1D || b == 0x1E) brk = 1;
    else if (b == 0xC2 && i + 1 < n && u[i + 1] == 0x85) brk = 2;
    else if (b == 0xE2 && i + 2 < n && u[i + 1] == 0x80 && (u[i + 2] == 0xA8 || u[i + 2] == 0xA9)) brk = 3;
    if (brk) {
      lines.push_back(s.substr(start, i - start));
      i += brk;
      start = i;
    } else {
      ++i;
    }
  }
  if (start < n) lines.push_back(s.substr(start));
  return lines;
}

std::string checksum_of(const std::string& key, const std::string& entry) {
  std::string body = "{\"entry\":" + entry + ",\"key\":" + key + "}";
  return sha256_hex((const uint8_t*)body.data(), body.size());
}

// ---------------------------------------------------------------- files

using Records = std::map<std::string, std::string>;  // canonical key -> canonical entry

// Records of a file's text; `ignored` counts the lines the rules above reject.
Records parse_file(const std::string& text, size_t& ignored) {
  Records out;
  ignored = 0;
  if (!valid_utf8(text)) return out;
  std::vector<std::string> lines = py_splitlines(text);
  if (lines.empty()) return out;
  if (py_strip(lines[0]) != kHeader) {
    ignored = lines.size();
    return out;
  }
  for (size_t i = 1; i < lines.size(); ++i) {
    if (py_strip(lines[i]).empty()) continue;
    Json rec;
    std::string err;
    bool ok = Parser(lines[i]).parse(rec, err) && rec.kind == Json::Object;
    const Json *key = nullptr, *entry = nullptr, *sum = nullptr;
    if (ok) {
      auto k = rec.members.find("key"), e = rec.members.find("entry"), c = rec.members.find("checksum");
      ok = k != rec.members.end() && e != rec.members.end() && c != rec.members.end();
      if (ok) {
        key = &k->second;
        entry = &e->second;
        sum = &c->second;
        ok = key->kind == Json::Object && entry->kind == Json::Object && sum->kind == Json::String;
      }
    }
    if (ok) {
      std::string ks, es;
      emit(ks, *key);
      emit(es, *entry);
      if (sum->text == checksum_of(ks, es)) {
        out[ks] = es;
        continue;
      }
    }
    ++ignored;
  }
  return out;
}

// Whole file, or false when it cannot be read (a missing file reads as empty).
bool read_file(const std::string& path, std::string& out) {
  out.clear();
  int fd = open(path.c_str(), O_RDONLY | O_CLOEXEC);
  if (fd < 0) return false;
  char buf[1 << 16];
  for (;;) {
    ssize_t n = read(fd, buf, sizeof buf);
    if (n < 0 && errno == EINTR) continue;
    if (n < 0) {
      close(fd);
      out.clear();
      return false;
    }
    if (n == 0) break;
    out.append(buf, (size_t)n);
  }
  close(fd);
  return true;
}

std::string parent_dir(const std::string& path) {
  size_t slash = path.find_last_of('/');
  if (slash == std::string::npos) return ".";
  if (slash == 0) return "/";
  return path.substr(0, slash);
}

tb_status io_error(const char* what, const std::string& path) {
  int e = errno;
  return tb::set_error(TB_ERR_IO, "tune", std::string(what) + " " + path + ": " + strerror(e) + " (errno " +
                                              std::to_string(e) + ")");
}

tb_status make_dirs(const std::string& dir) {
  if (dir.empty() || dir == "/" || dir == ".") return TB_OK;
  struct stat st;
  if (stat(dir.c_str(), &st) == 0) {
    if (S_ISDIR(st.st_mode)) return TB_OK;
    errno = ENOTDIR;
    return io_error("create directory", dir);
  }
  tb_status s = make_dirs(parent_dir(dir));
  if (s != TB_OK) return s;
  if (mkdir(dir.c_str(), 0777) != 0 && errno != EEXIST) return io_error("create directory", dir);
  return TB_OK;
}

bool write_all(int fd, const std::string& data) {
  size_t off = 0;
  while (off < data.size()) {
    ssize_t n = write(fd, data.data() + off, data.size() - off);
    if (n < 0 && errno == EINTR) continue;
    if (n <= 0) return false;
    off += (size_t)n;
  }
  return true;
}

// Copies text and a terminating NUL into out when it fits; *len always gets the length.
tb_status give_text(const std::string& text, char* out, size_t cap, size_t* len) {
  if (len) *len = text.size();
  if (!out || cap <= text.size())
    return tb::set_error(TB_ERR_INVALID, "tune",
                         "output buffer too small: " + std::to_string(text.size() + 1) + " bytes needed");
  memcpy(out, text.data(), text.size());
  out[text.size()] = '\0';
  return TB_OK;
}

bool object_json(const char* text, const char* what, std::string& out, tb_status& status) {
  std::string err;
  Json v;
  if (!text) {
    status = tb::set_error(TB_ERR_INVALID, "tune", std::string(what) + " is null");
    return false;
  }
  if (!canonical(text, out, err, &v) || v.kind != Json::Object) {
    status = tb::set_error(TB_ERR_INVALID, "tune",
                           std::string(what) + " is not a JSON object" + (err.empty() ? "" : ": " + err));
    return false;
  }
  return true;
}

}  // namespace

struct tb_tune_store {
  std::string path;
  mutable std::mutex mu;
  Records records;
  size_t ignored = 0;
  // Records by position for tb_tune_record, rebuilt after a change (under mu).
  mutable std::vector<Records::const_iterator> order;
  mutable bool order_stale = true;
};

extern "C" {

tb_status tb_tune_select(const tb_tune_measurement* ms, size_t n, size_t* winner) {
  if (!ms || !n || !winner) return tb::set_error(TB_ERR_INVALID, "tune", "select needs at least one measurement");
  uint64_t best = ms[0].median_ns;
  for (size_t i = 1; i < n; ++i) best = std::min(best, ms[i].median_ns);
  size_t w = n;
  for (size_t i = 0; i < n; ++i) {
    if ((double)ms[i].median_ns > (double)best * 1.02) continue;
    if (w == n) {
      w = i;
      continue;
    }
    const tb_tune_measurement &a = ms[i], &b = ms[w];
    const int names = strcmp(a.candidate ? a.candidate : "", b.candidate ? b.candidate : "");
    if (a.p95_ns != b.p95_ns ? a.p95_ns < b.p95_ns
                             : a.workspace_bytes != b.workspace_bytes ? a.workspace_bytes < b.workspace_bytes
                                                                      : names < 0)
      w = i;
  }
  *winner = w;
  return TB_OK;
}

tb_status tb_sha256_hex(const void* data, size_t len, char* out) {
  if (!out || (!data && len)) return tb::set_error(TB_ERR_INVALID, "tune", "null pointer");
  std::string h = sha256_hex((const uint8_t*)data, len);
  memcpy(out, h.c_str(), 65);
  return TB_OK;
}

tb_status tb_tune_canonical_json(const char* json, char* out, size_t cap, size_t* len) {
  if (!json) return tb::set_error(TB_ERR_INVALID, "tune", "json is null");
  std::string text, err;
  if (!canonical(json, text, err)) return tb::set_error(TB_ERR_INVALID, "tune", "not JSON: " + err);
  return give_text(text, out, cap, len);
}

tb_status tb_tune_open(const char* path, tb_tune_store** out) {
  if (!path || !*path || !out) return tb::set_error(TB_ERR_INVALID, "tune", "path and out are required");
  auto* s = new tb_tune_store();
  s->path = path;
  std::string text;
  if (read_file(s->path, text)) s->records = parse_file(text, s->ignored);
  *out = s;
  return TB_OK;
}

void tb_tune_release(tb_tune_store* store) { delete store; }

tb_status tb_tune_insert(tb_tune_store* store, const char* key_json, const char* entry_json) {
  if (!store) return tb::set_error(TB_ERR_INVALID, "tune", "store is null");
  std::string key, entry;
  tb_status st = TB_OK;
  if (!object_json(key_json, "key", key, st) || !object_json(entry_json, "entry", entry, st)) return st;
  std::lock_guard<std::mutex> g(store->mu);
  store->records[key] = entry;
  store->order_stale = true;
  return TB_OK;
}

tb_status tb_tune_get(const tb_tune_store* store, const char* key_json, char* entry, size_t cap, size_t* len) {
  if (!store) return tb::set_error(TB_ERR_INVALID, "tune", "store is null");
  std::string key;
  tb_status st = TB_OK;
  if (!object_json(key_json, "key", key, st)) return st;
  std::string found;
  {
    std::lock_guard<std::mutex> g(store->mu);
    auto it = store->records.find(key);
    if (it != store->records.end()) found = it->second;
  }
  if (found.empty()) {  // absent: an entry is never empty text
    if (len) *len = 0;
    if (entry && cap) entry[0] = '\0';
    return TB_OK;
  }
  return give_text(found, entry, cap, len);
}

tb_status tb_tune_stats(const tb_tune_store* store, size_t* records, size_t* ignored_lines) {
  if (!store) return tb::set_error(TB_ERR_INVALID, "tune", "store is null");
  std::lock_guard<std::mutex> g(store->mu);
  if (records) *records = store->records.size();
  if (ignored_lines) *ignored_lines = store->ignored;
  return TB_OK;
}

tb_status tb_tune_record(const tb_tune_store* store, size_t index, char* key, size_t key_cap, size_t* key_len,
                         char* entry, size_t entry_cap, size_t* entry_len) {
  if (!store) return tb::set_error(TB_ERR_INVALID, "tune", "store is null");
  std::string k, e;
  {
    std::lock_guard<std::mutex> g(store->mu);
    if (index >= store->records.size())
      return tb::set_error(TB_ERR_INVALID, "tune",
                           "record " + std::to_string(index) + " of " + std::to_string(store->records.size()));
    if (store->order_stale) {
      store->order.clear();
      for (auto it = store->records.begin(); it != store->records.end(); ++it) store->order.push_back(it);
      store->order_stale = false;
    }
    k = store->order[index]->first;
    e = store->order[index]->second;
  }
  tb_status a = give_text(k, key, key_cap, key_len);
  tb_status b = give_text(e, entry, entry_cap, entry_len);
  return a != TB_OK ? a : b;
}

tb_status tb_tune_flush(tb_tune_store* store) {
  if (!store) return tb::set_error(TB_ERR_INVALID, "tune", "store is null");
  std::lock_guard<std::mutex> g(store->mu);
  const std::string& path = store->path;
  std::string dir = parent_dir(path);
  tb_status st = make_dirs(dir);
  if (st != TB_OK) return st;
  std::string lock_path = path + ".lock", tmp_path = path + ".tmp";
  int lock = open(lock_path.c_str(), O_RDWR | O_CREAT | O_APPEND | O_CLOEXEC, 0666);
  if (lock < 0) return io_error("open", lock_path);
  int r;
  do r = flock(lock, LOCK_EX); while (r != 0 && errno == EINTR);
  if (r != 0) {
    st = io_error("lock", lock_path);
    close(lock);
    return st;
  }
  // Under the lock: merge with the file (this store's records win), write, rename.
  std::string text;
  Records merged;
  size_t ignored = 0;
  if (read_file(path, text)) merged = parse_file(text, ignored);
  for (const auto& kv : store->records) merged[kv.first] = kv.second;
  std::vector<std::string> rows;
  rows.reserve(merged.size());
  for (const auto& kv : merged)
    rows.push_back("{\"checksum\":\"" + checksum_of(kv.first, kv.second) + "\",\"entry\":" + kv.second +
                   ",\"key\":" + kv.first + "}");
  std::sort(rows.begin(), rows.end());
  std::string content = std::string(kHeader) + "\n";
  for (const auto& row : rows) content += row + "\n";
  bool renamed = false;
  int fd = open(tmp_path.c_str(), O_WRONLY | O_CREAT | O_TRUNC | O_CLOEXEC, 0666);
  if (fd < 0) {
    st = io_error("open", tmp_path);
  } else if (!write_all(fd, content)) {
    st = io_error("write", tmp_path);
    close(fd);
  } else if (fsync(fd) != 0) {
    st = io_error("fsync", tmp_path);
    close(fd);
  } else if (close(fd) != 0) {
    st = io_error("close", tmp_path);
  } else if (rename(tmp_path.c_str(), path.c_str()) != 0) {
    st = io_error("rename", tmp_path);
  } else {
    renamed = true;
    int dfd = open(dir.c_str(), O_RDONLY | O_CLOEXEC);
    if (dfd >= 0) {
      // Some file systems refuse fsync on a directory; the rename is still in place.
      if (fsync(dfd) != 0 && errno != EINVAL && errno != EBADF) st = io_error("fsync", dir);
      close(dfd);
    }
  }
  if (renamed) {  // the merged records are the file now, even if the directory fsync failed
    store->records = std::move(merged);
    store->ignored = ignored;
    store->order_stale = true;
  } else if (fd >= 0) {
    unlink(tmp_path.c_str());  // the file on disk is untouched; leave no partial copy beside it
  }
  flock(lock, LOCK_UN);
  close(lock);
  return st;
}

}  // extern "C"
