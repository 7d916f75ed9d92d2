// The systems layer of the core C ABI that compiled programs call for what a
// standard library provides: files and directories, environment, processes,
// OS threads, atomics, a cooperative executor for poll-based futures, a
// small JIT page allocator, and handle-based containers (growable i64 / f32
// vectors, byte strings, an i64 hash map, reference-counted and boxed i64
// cells, lazy vector iterators, FIFO channels).
//
// Conventions, as in the rest of the ABI: paths and commands are
// NUL-terminated C strings; container handles are table slots counted from 0
// (a freed slot is reused); getters return 0 and mutators -1 on a bad handle.
// Each table has its own mutex, so containers may be used from several threads.
//
// Names, argument orders and return conventions follow the reference's
// exports (runtime/src/lib.rs:856-1200, 1407-1780, 4020-4998); the code is this
// library's own.
#include <dirent.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <sys/wait.h>
#include <unistd.h>

#include <atomic>
#include <cerrno>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <deque>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

extern "C" {
int64_t aether_alloc_bytes(int64_t n);
}

namespace {

// A table of optional objects addressed by slot; free slots are reused.
template <class T>
struct Table {
  std::mutex mu;
  std::vector<std::unique_ptr<T>> slots;
  int64_t put(std::unique_ptr<T> v) {
    std::lock_guard<std::mutex> l(mu);
    for (size_t i = 0; i < slots.size(); ++i)
      if (!slots[i]) {
        slots[i] = std::move(v);
        return (int64_t)i;
      }
    slots.push_back(std::move(v));
    return (int64_t)slots.size() - 1;
  }
  T* get(int64_t h) {
    std::lock_guard<std::mutex> l(mu);
    return (h >= 0 && (size_t)h < slots.size()) ? slots[h].get() : nullptr;
  }
  bool drop(int64_t h) {
    std::lock_guard<std::mutex> l(mu);
    if (h < 0 || (size_t)h >= slots.size() || !slots[h]) return false;
    slots[h].reset();
    return true;
  }
};

struct VecI64 {
  std::vector<int64_t> v;
};
struct VecF32 {
  std::vector<float> v;
};
struct Str {
  std::string s;
};
struct Map {
  std::unordered_map<int64_t, int64_t> m;
};
struct Rc {
  int64_t value;
  int64_t count;
};
struct BoxI {
  int64_t value;
};
struct Chan {
  std::mutex mu;
  std::deque<int64_t> q;
};
// A lazy iterator node: a source vector, or an adapter over another iterator.
struct Iter {
  enum Kind { Source, MapDouble, FilterPositive, Take } kind;
  int64_t vec = -1;    // Source: vector handle
  size_t pos = 0;      // Source: next index
  int64_t inner = -1;  // adapters: the iterator they pull from
  int64_t left = 0;    // Take: items still allowed
};

Table<VecI64> g_vi;
Table<VecF32> g_vf;
Table<Str> g_str;
Table<Map> g_map;
Table<Rc> g_rc;
Table<BoxI> g_box;
Table<Chan> g_chan;
Table<Iter> g_iter;
thread_local int64_t t_last_file_size = 0;

bool cstr(int64_t p, std::string* out) {
  if (!p) return false;
  *out = (const char*)p;
  return true;
}

bool iter_next(int64_t h, int64_t* out) {
  Iter* it = g_iter.get(h);
  if (!it) return false;
  switch (it->kind) {
    case Iter::Source: {
      VecI64* v = g_vi.get(it->vec);
      if (!v || it->pos >= v->v.size()) return false;
      *out = v->v[it->pos++];
      return true;
    }
    case Iter::MapDouble:
      if (!iter_next(it->inner, out)) return false;
      *out *= 2;
      return true;
    case Iter::FilterPositive:
      while (iter_next(it->inner, out))
        if (*out > 0) return true;
      return false;
    case Iter::Take:
      if (it->left <= 0 || !iter_next(it->inner, out)) return false;
      --it->left;
      return true;
  }
  return false;
}

int64_t iter_adapter(Iter::Kind k, int64_t inner, int64_t left = 0) {
  if (!g_iter.get(inner)) return -1;
  auto it = std::make_unique<Iter>();
  it->kind = k;
  it->inner = inner;
  it->left = left;
  return g_iter.put(std::move(it));
}

typedef int64_t (*Fn1)(int64_t);
typedef int64_t (*Fn0)();

struct Job {  // one spawned thread and the value its function returned
  std::thread t;
  int64_t result = 0;
};

}  // namespace

extern "C" {

// ================================================================================================ files
int64_t aether_read_file(int64_t path) {
  std::string p;
  if (!cstr(path, &p)) return 0;
  FILE* f = fopen(p.c_str(), "rb");
  if (!f) return 0;
  std::vector<char> buf;
  char chunk[65536];
  size_t n;
  while ((n = fread(chunk, 1, sizeof(chunk), f)) > 0) buf.insert(buf.end(), chunk, chunk + n);
  const bool err = ferror(f);
  fclose(f);
  if (err) return 0;
  const int64_t out = aether_alloc_bytes((int64_t)std::max<size_t>(buf.size(), 1));  // freed by aether_free_bytes
  if (!out) return 0;
  if (!buf.empty()) memcpy((void*)out, buf.data(), buf.size());
  t_last_file_size = (int64_t)buf.size();
  return out;
}
int64_t aether_file_size_last() { return t_last_file_size; }
int aether_write_file(int64_t path, int64_t buf, int64_t n) {
  std::string p;
  if (!cstr(path, &p) || n < 0 || (n > 0 && !buf)) return -1;
  FILE* f = fopen(p.c_str(), "wb");
  if (!f) return -1;
  const bool ok = n == 0 || fwrite((const void*)buf, 1, (size_t)n, f) == (size_t)n;
  return (fclose(f) == 0 && ok) ? 0 : -1;
}
int64_t aether_file_size(int64_t path) {
  std::string p;
  struct stat st;
  if (!cstr(path, &p) || stat(p.c_str(), &st) != 0) return -1;
  return (int64_t)st.st_size;
}
int64_t aether_path_exists(int64_t path) {
  std::string p;
  struct stat st;
  return cstr(path, &p) && stat(p.c_str(), &st) == 0;
}
int64_t aether_is_dir(int64_t path) {
  std::string p;
  struct stat st;
  return cstr(path, &p) && stat(p.c_str(), &st) == 0 && S_ISDIR(st.st_mode);
}
int aether_create_dir_all(int64_t path) {
  std::string p;
  if (!cstr(path, &p) || p.empty()) return -1;
  for (size_t i = 1; i <= p.size(); ++i) {
    if (i == p.size() || p[i] == '/') {
      const std::string part = p.substr(0, i);
      if (mkdir(part.c_str(), 0755) != 0 && errno != EEXIST) return -1;
    }
  }
  return aether_is_dir(path) ? 0 : -1;
}
int aether_remove_file(int64_t path) {
  std::string p;
  return (cstr(path, &p) && unlink(p.c_str()) == 0) ? 0 : -1;
}
int aether_rename(int64_t src, int64_t dst) {
  std::string s, d;
  return (cstr(src, &s) && cstr(dst, &d) && rename(s.c_str(), d.c_str()) == 0) ? 0 : -1;
}
int64_t aether_copy_file(int64_t src, int64_t dst) {
  std::string s, d;
  if (!cstr(src, &s) || !cstr(dst, &d)) return -1;
  FILE* in = fopen(s.c_str(), "rb");
  if (!in) return -1;
  FILE* out = fopen(d.c_str(), "wb");
  if (!out) {
    fclose(in);
    return -1;
  }
  char chunk[65536];
  size_t n;
  int64_t total = 0;
  bool ok = true;
  while ((n = fread(chunk, 1, sizeof(chunk), in)) > 0) {
    if (fwrite(chunk, 1, n, out) != n) {
      ok = false;
      break;
    }
    total += (int64_t)n;
  }
  ok = ok && !ferror(in);
  fclose(in);
  ok = (fclose(out) == 0) && ok;
  return ok ? total : -1;
}
// Entries of a directory, "." and ".." excluded; -1 when it cannot be read.
int64_t aether_read_dir_count(int64_t path) {
  std::string p;
  if (!cstr(path, &p)) return -1;
  DIR* d = opendir(p.c_str());
  if (!d) return -1;
  int64_t n = 0;
  while (struct dirent* e = readdir(d))
    if (strcmp(e->d_name, ".") && strcmp(e->d_name, "..")) ++n;
  closedir(d);
  return n;
}

// ================================================================================================ env, process
void aether_env_set(int64_t key, int64_t val) {
  std::string k, v;
  if (cstr(key, &k) && cstr(val, &v)) setenv(k.c_str(), v.c_str(), 1);
}
// The variable parsed as a decimal integer; -1 when unset or not an integer.
int64_t aether_env_var_i64(int64_t key) {
  std::string k;
  if (!cstr(key, &k)) return -1;
  const char* v = getenv(k.c_str());
  if (!v) return -1;
  char* end = nullptr;
  errno = 0;
  const long long x = strtoll(v, &end, 10);
  while (end && (*end == ' ' || *end == '\n' || *end == '\t')) ++end;
  return (errno || end == v || (end && *end)) ? -1 : (int64_t)x;
}
// `sh -c cmd`; the exit code, or -1 when it could not run or ended on a signal.
int64_t aether_process_run(int64_t cmd) {
  std::string c;
  if (!cstr(cmd, &c)) return -1;
  fflush(stdout);
  const pid_t pid = fork();
  if (pid < 0) return -1;
  if (pid == 0) {
    execl("/bin/sh", "sh", "-c", c.c_str(), (char*)nullptr);
    _exit(127);
  }
  int st = 0;
  while (waitpid(pid, &st, 0) < 0)
    if (errno != EINTR) return -1;
  return WIFEXITED(st) ? WEXITSTATUS(st) : -1;
}

// ================================================================================================ threads, atomics, async
// Runs fn(arg) on a new OS thread; join returns its result and consumes the handle.
int64_t aether_thread_spawn(int64_t fn_ptr, int64_t arg) {
  if (!fn_ptr) return 0;
  auto* job = new Job;
  try {
    job->t = std::thread([job, fn_ptr, arg] { job->result = ((Fn1)fn_ptr)(arg); });
  } catch (...) {
    delete job;
    return 0;
  }
  return (int64_t)job;
}
int64_t aether_thread_join(int64_t handle) {
  if (!handle) return 0;
  auto* job = (Job*)handle;
  job->t.join();
  const int64_t r = job->result;
  delete job;
  return r;
}
int64_t aether_atomic_load_i64(int64_t addr) {
  return __atomic_load_n((int64_t*)addr, __ATOMIC_SEQ_CST);
}
void aether_atomic_store_i64(int64_t addr, int64_t v) { __atomic_store_n((int64_t*)addr, v, __ATOMIC_SEQ_CST); }
// Returns the previous value.
int64_t aether_atomic_fetch_add_i64(int64_t addr, int64_t v) {
  return __atomic_fetch_add((int64_t*)addr, v, __ATOMIC_SEQ_CST);
}
// Returns the value found; the swap happened when it equals `expected`.
int64_t aether_atomic_cas_i64(int64_t addr, int64_t expected, int64_t desired) {
  int64_t e = expected;
  __atomic_compare_exchange_n((int64_t*)addr, &e, desired, false, __ATOMIC_SEQ_CST, __ATOMIC_SEQ_CST);
  return e;
}
// A future is [poll_fn, state..., result at slot 2]: poll until it returns
// nonzero, then hand back slot 2.
int64_t aether_block_on(int64_t fut) {
  if (!fut) return 0;
  int64_t* f = (int64_t*)fut;
  if (f[0]) {
    Fn1 poll = (Fn1)f[0];
    while (poll(fut) == 0) {
    }
  }
  return f[2];
}
// Round-robin over (poll_fn, state) pairs until every task reports ready;
// returns the number of polls made.
int64_t aether_executor_run(int64_t tasks, int64_t n) {
  if (!tasks || n <= 0) return 0;
  const int64_t* t = (const int64_t*)tasks;
  std::vector<char> done((size_t)n, 0);
  int64_t left = n, polls = 0;
  while (left > 0) {
    for (int64_t i = 0; i < n; ++i) {
      if (done[i]) continue;
      if (!t[2 * i]) {
        done[i] = 1;
        --left;
        continue;
      }
      ++polls;
      if (((Fn1)t[2 * i])(t[2 * i + 1]) != 0) {
        done[i] = 1;
        --left;
      }
    }
  }
  return polls;
}

// ================================================================================================ JIT pages
// Read-write-execute pages for generated code, called as fn() -> i64.
int64_t aether_alloc_executable(int64_t n) {
  if (n <= 0) return 0;
  void* p = mmap(nullptr, (size_t)n, PROT_READ | PROT_WRITE | PROT_EXEC, MAP_PRIVATE | MAP_ANONYMOUS, -1, 0);
  return p == MAP_FAILED ? 0 : (int64_t)p;
}
void aether_free_executable(int64_t p, int64_t n) {
  if (p && n > 0) munmap((void*)p, (size_t)n);
}
int64_t aether_call_jit_i64(int64_t p) {
  if (!p) return 0;
  __builtin___clear_cache((char*)p, (char*)p + 4096);
  return ((Fn0)p)();
}
// n f32 values in [0, 4) from a multiplicative-hash ramp of `seed` (a test
// input for vectorised dot products); freed with aether_free_bytes.
int64_t aether_avx2_witness_arr(int64_t seed, int64_t n) {
  if (n <= 0) return 0;
  const int64_t p = aether_alloc_bytes(n * 4);
  if (!p) return 0;
  uint32_t s = (uint32_t)seed;
  for (int64_t i = 0; i < n; ++i) {
    s = s * 2654435761u + 0x9E37u;
    const uint32_t bits = 0x3F800000u | ((s >> 9) & 0x7FFFFFu);  // [1, 2)
    float v;
    memcpy(&v, &bits, 4);
    ((float*)p)[i] = v - 1.f + (float)(i & 7) * 0.25f;
  }
  return p;
}
// Calling-convention probes for generated code.
float aether_test_add_f32(float a, float b) { return a + b; }
double aether_test_add_f64(double a, double b) { return a + b; }
int64_t aether_test_f32_to_i64(float x) { return (int64_t)x; }
int64_t aether_test_f64_to_i64(double x) { return (int64_t)x; }
float aether_test_mix_if(int i, float f, int j) { return (float)(i + j) * f; }

// ================================================================================================ vectors
int64_t aether_vec_i64_new() { return g_vi.put(std::make_unique<VecI64>()); }
int aether_vec_i64_free(int64_t h) { return g_vi.drop(h) ? 0 : -1; }
int aether_vec_i64_push(int64_t h, int64_t v) {
  VecI64* x = g_vi.get(h);
  if (!x) return -1;
  x->v.push_back(v);
  return 0;
}
int64_t aether_vec_i64_len(int64_t h) {
  VecI64* x = g_vi.get(h);
  return x ? (int64_t)x->v.size() : 0;
}
int64_t aether_vec_i64_get(int64_t h, int64_t i) {
  VecI64* x = g_vi.get(h);
  return (x && i >= 0 && (size_t)i < x->v.size()) ? x->v[i] : 0;
}
int aether_vec_i64_set(int64_t h, int64_t i, int64_t v) {
  VecI64* x = g_vi.get(h);
  if (!x || i < 0 || (size_t)i >= x->v.size()) return -1;
  x->v[i] = v;
  return 0;
}
// Valid until the next push (growth may move the storage).
int64_t aether_vec_i64_as_ptr(int64_t h) {
  VecI64* x = g_vi.get(h);
  return x ? (int64_t)x->v.data() : 0;
}
int64_t aether_vec_f32_new() { return g_vf.put(std::make_unique<VecF32>()); }
int aether_vec_f32_free(int64_t h) { return g_vf.drop(h) ? 0 : -1; }
// `bits` carries the float's bit pattern in its low 32 bits.
int aether_vec_f32_push(int64_t h, int64_t bits) {
  VecF32* x = g_vf.get(h);
  if (!x) return -1;
  const uint32_t b = (uint32_t)bits;
  float f;
  memcpy(&f, &b, 4);
  x->v.push_back(f);
  return 0;
}
int64_t aether_vec_f32_len(int64_t h) {
  VecF32* x = g_vf.get(h);
  return x ? (int64_t)x->v.size() : 0;
}
int64_t aether_vec_f32_as_ptr(int64_t h) {
  VecF32* x = g_vf.get(h);
  return x ? (int64_t)x->v.data() : 0;
}

// ================================================================================================ strings
int64_t aether_string_new() { return g_str.put(std::make_unique<Str>()); }
int aether_string_free(int64_t h) { return g_str.drop(h) ? 0 : -1; }
int aether_string_push_byte(int64_t h, int64_t b) {
  Str* s = g_str.get(h);
  if (!s) return -1;
  s->s.push_back((char)(uint8_t)b);
  return 0;
}
int64_t aether_string_len(int64_t h) {
  Str* s = g_str.get(h);
  return s ? (int64_t)s->s.size() : 0;
}
int64_t aether_string_byte_at(int64_t h, int64_t i) {
  Str* s = g_str.get(h);
  return (s && i >= 0 && (size_t)i < s->s.size()) ? (uint8_t)s->s[i] : 0;
}
// NUL-terminated view, valid until the next push.
int64_t aether_string_as_ptr(int64_t h) {
  Str* s = g_str.get(h);
  return s ? (int64_t)s->s.c_str() : 0;
}

// ================================================================================================ hash map
int64_t aether_hashmap_i64_new() { return g_map.put(std::make_unique<Map>()); }
int aether_hashmap_i64_free(int64_t h) { return g_map.drop(h) ? 0 : -1; }
int aether_hashmap_i64_insert(int64_t h, int64_t k, int64_t v) {
  Map* m = g_map.get(h);
  if (!m) return -1;
  m->m[k] = v;
  return 0;
}
int64_t aether_hashmap_i64_get(int64_t h, int64_t k) {
  Map* m = g_map.get(h);
  if (!m) return 0;
  auto it = m->m.find(k);
  return it == m->m.end() ? 0 : it->second;
}
int64_t aether_hashmap_i64_contains(int64_t h, int64_t k) {
  Map* m = g_map.get(h);
  return m && m->m.count(k);
}
// The removed value, or 0 when the key was absent.
int64_t aether_hashmap_i64_remove(int64_t h, int64_t k) {
  Map* m = g_map.get(h);
  if (!m) return 0;
  auto it = m->m.find(k);
  if (it == m->m.end()) return 0;
  const int64_t v = it->second;
  m->m.erase(it);
  return v;
}
int64_t aether_hashmap_i64_len(int64_t h) {
  Map* m = g_map.get(h);
  return m ? (int64_t)m->m.size() : 0;
}

// ================================================================================================ rc / box cells
int64_t aether_rc_i64_new(int64_t v) { return g_rc.put(std::make_unique<Rc>(Rc{v, 1})); }
int64_t aether_rc_i64_clone(int64_t h) {
  Rc* r = g_rc.get(h);
  if (!r) return -1;
  ++r->count;
  return h;  // clones share the slot
}
int aether_rc_i64_drop(int64_t h) {
  Rc* r = g_rc.get(h);
  if (!r) return -1;
  if (--r->count <= 0) g_rc.drop(h);
  return 0;
}
int64_t aether_rc_i64_get(int64_t h) {
  Rc* r = g_rc.get(h);
  return r ? r->value : 0;
}
int64_t aether_rc_i64_strong_count(int64_t h) {
  Rc* r = g_rc.get(h);
  return r ? r->count : 0;
}
int64_t aether_box_i64_new(int64_t v) { return g_box.put(std::make_unique<BoxI>(BoxI{v})); }
int aether_box_i64_free(int64_t h) { return g_box.drop(h) ? 0 : -1; }
int64_t aether_box_i64_get(int64_t h) {
  BoxI* b = g_box.get(h);
  return b ? b->value : 0;
}
int aether_box_i64_set(int64_t h, int64_t v) {
  BoxI* b = g_box.get(h);
  if (!b) return -1;
  b->value = v;
  return 0;
}

// ================================================================================================ channels
int64_t aether_chan_i64_new() { return g_chan.put(std::make_unique<Chan>()); }
int aether_chan_i64_free(int64_t h) { return g_chan.drop(h) ? 0 : -1; }
int aether_chan_i64_send(int64_t h, int64_t v) {
  Chan* c = g_chan.get(h);
  if (!c) return -1;
  std::lock_guard<std::mutex> l(c->mu);
  c->q.push_back(v);
  return 0;
}
// Non-blocking: 1 and the value through out_ptr, or 0 when empty.
int aether_chan_i64_recv(int64_t h, int64_t out_ptr) {
  Chan* c = g_chan.get(h);
  if (!c || !out_ptr) return 0;
  std::lock_guard<std::mutex> l(c->mu);
  if (c->q.empty()) return 0;
  *(int64_t*)out_ptr = c->q.front();
  c->q.pop_front();
  return 1;
}
int64_t aether_chan_i64_len(int64_t h) {
  Chan* c = g_chan.get(h);
  if (!c) return 0;
  std::lock_guard<std::mutex> l(c->mu);
  return (int64_t)c->q.size();
}

// ================================================================================================ iterators
int64_t aether_iter_vec_i64_new(int64_t vec) {
  if (!g_vi.get(vec)) return -1;
  auto it = std::make_unique<Iter>();
  it->kind = Iter::Source;
  it->vec = vec;
  return g_iter.put(std::move(it));
}
int aether_iter_vec_i64_free(int64_t h) { return g_iter.drop(h) ? 0 : -1; }
// 1 and the value through out_value, 0 when exhausted, -1 on bad arguments.
int64_t aether_iter_vec_i64_next(int64_t h, int64_t out_value) {
  if (!out_value || !g_iter.get(h)) return -1;
  int64_t v;
  if (!iter_next(h, &v)) return 0;
  *(int64_t*)out_value = v;
  return 1;
}
int64_t aether_iter_vec_i64_map_double(int64_t h) { return iter_adapter(Iter::MapDouble, h); }
int64_t aether_iter_vec_i64_filter_positive(int64_t h) { return iter_adapter(Iter::FilterPositive, h); }
int64_t aether_iter_vec_i64_take(int64_t h, int64_t n) { return iter_adapter(Iter::Take, h, n); }
// Drains the iterator into a new vector and returns its handle.
int64_t aether_iter_vec_i64_collect(int64_t h) {
  if (!g_iter.get(h)) return -1;
  const int64_t v = aether_vec_i64_new();
  int64_t x;
  while (iter_next(h, &x)) aether_vec_i64_push(v, x);
  return v;
}
int64_t aether_iter_vec_i64_fold_sum(int64_t h) {
  int64_t s = 0, x;
  while (iter_next(h, &x)) s += x;
  return s;
}

}  // extern "C"
