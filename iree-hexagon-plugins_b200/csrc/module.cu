// Loader and invoker of executables compiled by hxb_compile_mlir
// (include/hxb200_compiler.h): the B200 counterpart of loading a .vmfb's
// hal.executable and running one of its functions (iree-run-module).
//
// Each function becomes one HAL command buffer recorded once at load time.
// Its bindings are binding-table slots -- arguments first, then results,
// then the function's transient buffers -- so an invocation only supplies a
// table of the caller's buffers (plus the module's transients) to
// hxb_hal_device_queue_execute; the command buffer is captured as a CUDA
// graph at its first invocation and updated in place when later ones bind
// other buffers.
#include <stdlib.h>
#include <string.h>

#include <new>
#include <string>
#include <vector>

#include "hxb200_compiler.h"
#include "runtime_common.h"

namespace {

using hxb::fail;

struct Binding {
  uint32_t kind, index;
  uint64_t offset, length;
};
struct Dispatch {
  uint32_t ordinal;
  std::vector<uint32_t> constants;
  std::vector<Binding> bindings;
};
struct Function {
  std::string name;
  std::vector<hxb_tensor_desc_t> args, results;
  std::vector<uint64_t> transient_bytes;
  std::vector<hxb_hal_buffer_t*> transients;
  std::vector<Dispatch> dispatches;
  hxb_hal_command_buffer_t* cb = nullptr;
};

class Reader {
 public:
  Reader(const uint8_t* p, size_t n) : p_(p), n_(n) {}
  bool u32(uint32_t* v) {
    if (n_ - i_ < 4) return false;
    *v = 0;
    for (int k = 0; k < 4; ++k) *v |= (uint32_t)p_[i_ + k] << (8 * k);
    i_ += 4;
    return true;
  }
  bool u64(uint64_t* v) {
    if (n_ - i_ < 8) return false;
    *v = 0;
    for (int k = 0; k < 8; ++k) *v |= (uint64_t)p_[i_ + k] << (8 * k);
    i_ += 8;
    return true;
  }
  bool str(std::string* s) {
    uint32_t len = 0;
    if (!u32(&len) || n_ - i_ < len) return false;
    s->assign(reinterpret_cast<const char*>(p_ + i_), len);
    i_ += len;
    return true;
  }
  bool bytes(size_t n, const void* want) {
    if (n_ - i_ < n || memcmp(p_ + i_, want, n) != 0) return false;
    i_ += n;
    return true;
  }

 private:
  const uint8_t* p_;
  size_t n_, i_ = 0;
};

uint64_t desc_bytes(const hxb_tensor_desc_t& d) {
  uint64_t n = d.element_type == HXB_ELEMENT_F32 ? 4 : d.element_type == HXB_ELEMENT_F16 ? 2 : 1;
  for (int i = 0; i < d.rank; ++i) n *= (uint64_t)d.dims[i];
  return n;
}

bool read_descs(Reader& r, std::vector<hxb_tensor_desc_t>* out) {
  uint32_t n = 0;
  if (!r.u32(&n) || n > 4096) return false;
  for (uint32_t i = 0; i < n; ++i) {
    hxb_tensor_desc_t d{};
    uint32_t e = 0, rank = 0;
    if (!r.u32(&e) || !r.u32(&rank) || rank > HXB_MAX_RANK || e > HXB_ELEMENT_I8) return false;
    d.element_type = (int32_t)e;
    d.rank = (int32_t)rank;
    for (uint32_t k = 0; k < rank; ++k) {
      uint64_t x = 0;
      if (!r.u64(&x) || x > (1ull << 40)) return false;
      d.dims[k] = (int64_t)x;
    }
    out->push_back(d);
  }
  return true;
}

}  // namespace

struct hxb_module_s {
  hxb_hal_device_t* device = nullptr;
  std::vector<Function> functions;
};

namespace {

Function* find(hxb_module_t* m, const char* name) {
  if (!m || !name) return nullptr;
  for (Function& f : m->functions)
    if (f.name == name) return &f;
  // "main" also names "main$async" (the coarse-fences body of an IREE entry)
  for (Function& f : m->functions)
    if (f.name == std::string(name) + "$async") return &f;
  return nullptr;
}

void destroy(hxb_module_t* m) {
  for (Function& f : m->functions) {
    if (f.cb) hxb_hal_command_buffer_release(f.cb);
    for (hxb_hal_buffer_t* b : f.transients) hxb_hal_buffer_release(b);
  }
  delete m;
}

}  // namespace

extern "C" hxb_status_t hxb_module_load(hxb_hal_device_t* device, const void* executable,
                                        size_t size, hxb_module_t** out_module) {
  if (!device || !executable || !out_module)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "module_load: null argument");
  *out_module = nullptr;
  Reader r(static_cast<const uint8_t*>(executable), size);
  uint32_t version = 0, nf = 0;
  std::string format;
  if (!r.bytes(4, "HXBX") || !r.u32(&version) || version != 1 || !r.str(&format) ||
      format != HXB_EXECUTABLE_FORMAT || !r.u32(&nf) || nf > 4096)
    return fail(HXB_STATUS_INVALID_ARGUMENT,
                "module_load: not an executable of format %s (version 1)", HXB_EXECUTABLE_FORMAT);
  hxb_module_t* m = new (std::nothrow) hxb_module_s();
  if (!m) return fail(HXB_STATUS_RESOURCE_EXHAUSTED, "module_load: out of host memory");
  m->device = device;
  m->functions.resize(nf);
  bool ok = true;
  for (uint32_t i = 0; i < nf && ok; ++i) {
    Function& f = m->functions[i];
    uint32_t nt = 0, nd = 0;
    ok = r.str(&f.name) && read_descs(r, &f.args) && read_descs(r, &f.results) && r.u32(&nt) &&
         nt <= 4096;
    for (uint32_t t = 0; ok && t < nt; ++t) {
      uint64_t b = 0;
      ok = r.u64(&b);
      f.transient_bytes.push_back(b);
    }
    ok = ok && r.u32(&nd) && nd <= (1u << 20);
    for (uint32_t d = 0; ok && d < nd; ++d) {
      Dispatch x;
      uint32_t nc = 0, nb = 0;
      ok = r.u32(&x.ordinal) && r.u32(&nc) && nc <= 64;
      for (uint32_t c = 0; ok && c < nc; ++c) {
        uint32_t v = 0;
        ok = r.u32(&v);
        x.constants.push_back(v);
      }
      ok = ok && r.u32(&nb) && nb <= 255;
      for (uint32_t b = 0; ok && b < nb; ++b) {
        Binding y{};
        ok = r.u32(&y.kind) && r.u32(&y.index) && r.u64(&y.offset) && r.u64(&y.length) &&
             y.kind <= 2;
        x.bindings.push_back(y);
      }
      f.dispatches.push_back(std::move(x));
    }
  }
  if (!ok) {
    destroy(m);
    return fail(HXB_STATUS_INVALID_ARGUMENT, "module_load: truncated or malformed executable");
  }
  // transients, and one command buffer per function over table slots
  for (Function& f : m->functions) {
    const uint32_t na = (uint32_t)f.args.size(), nr = (uint32_t)f.results.size();
    for (uint64_t b : f.transient_bytes) {
      hxb_hal_buffer_t* buf = nullptr;
      hxb_status_t s = hxb_hal_buffer_allocate(device, b ? b : 16, &buf);
      if (s != HXB_OK) {
        destroy(m);
        return s;
      }
      f.transients.push_back(buf);
    }
    const uint32_t cap = na + nr + (uint32_t)f.transients.size();
    hxb_status_t s = hxb_hal_command_buffer_create(device, cap, &f.cb);
    if (s == HXB_OK) s = hxb_hal_command_buffer_begin(f.cb);
    for (size_t d = 0; s == HXB_OK && d < f.dispatches.size(); ++d) {
      const Dispatch& x = f.dispatches[d];
      std::vector<hxb_hal_buffer_ref_t> refs;
      for (const Binding& b : x.bindings) {
        const uint32_t base = b.kind == 0 ? 0 : b.kind == 1 ? na : na + nr;
        const uint32_t limit = b.kind == 0 ? na : b.kind == 1 ? nr : (uint32_t)f.transients.size();
        if (b.index >= limit) {
          s = fail(HXB_STATUS_INVALID_ARGUMENT, "module_load: @%s dispatch %zu binds slot %u of %u",
                   f.name.c_str(), d, b.index, limit);
          break;
        }
        refs.push_back(hxb_hal_buffer_ref_t{nullptr, b.offset, b.length, base + b.index, 0});
      }
      if (s == HXB_OK)
        s = hxb_hal_command_buffer_dispatch(f.cb, x.ordinal, x.constants.data(),
                                            (uint32_t)x.constants.size(), refs.data(),
                                            (uint32_t)refs.size());
    }
    if (s == HXB_OK) s = hxb_hal_command_buffer_end(f.cb);
    if (s != HXB_OK) {
      destroy(m);
      return s;
    }
  }
  *out_module = m;
  return HXB_OK;
}

extern "C" void hxb_module_release(hxb_module_t* module) {
  if (module) destroy(module);
}

extern "C" int32_t hxb_module_function_count(hxb_module_t* module) {
  return module ? (int32_t)module->functions.size() : 0;
}

extern "C" const char* hxb_module_function_name(hxb_module_t* module, int32_t index) {
  if (!module || index < 0 || index >= (int32_t)module->functions.size()) return nullptr;
  return module->functions[index].name.c_str();
}

extern "C" hxb_status_t hxb_module_signature(hxb_module_t* module, const char* name,
                                             int32_t* n_args, int32_t* n_results,
                                             hxb_tensor_desc_t* descs, int32_t capacity) {
  Function* f = find(module, name);
  if (!f) return fail(HXB_STATUS_INVALID_ARGUMENT, "module_signature: no function '%s'", name ? name : "");
  if (n_args) *n_args = (int32_t)f->args.size();
  if (n_results) *n_results = (int32_t)f->results.size();
  int32_t k = 0;
  for (const auto* list : {&f->args, &f->results})
    for (const hxb_tensor_desc_t& d : *list) {
      if (descs && k < capacity) descs[k] = d;
      ++k;
    }
  return HXB_OK;
}

extern "C" int32_t hxb_module_dispatch_count(hxb_module_t* module, const char* name) {
  Function* f = find(module, name);
  return f ? (int32_t)f->dispatches.size() : -1;
}

extern "C" hxb_status_t hxb_module_invoke(hxb_module_t* module, const char* name,
                                          const hxb_hal_buffer_binding_t* args, uint32_t n_args,
                                          const hxb_hal_buffer_binding_t* results,
                                          uint32_t n_results, hxb_hal_semaphore_t* wait_semaphore,
                                          uint64_t wait_value,
                                          hxb_hal_semaphore_t* signal_semaphore,
                                          uint64_t signal_value) {
  Function* f = find(module, name);
  if (!f) return fail(HXB_STATUS_INVALID_ARGUMENT, "module_invoke: no function '%s'", name ? name : "");
  if (n_args != f->args.size() || n_results != f->results.size() ||
      (n_args && !args) || (n_results && !results))
    return fail(HXB_STATUS_INVALID_ARGUMENT,
                "module_invoke: @%s takes %zu argument(s) and %zu result(s), got %u and %u",
                f->name.c_str(), f->args.size(), f->results.size(), n_args, n_results);
  std::vector<hxb_hal_buffer_binding_t> table;
  for (uint32_t i = 0; i < n_args + n_results; ++i) {
    const bool is_arg = i < n_args;
    const hxb_hal_buffer_binding_t& b = is_arg ? args[i] : results[i - n_args];
    const hxb_tensor_desc_t& d = is_arg ? f->args[i] : f->results[i - n_args];
    if (b.length < desc_bytes(d))
      return fail(HXB_STATUS_INVALID_ARGUMENT,
                  "module_invoke: @%s %s %u binds %llu bytes, needs %llu", f->name.c_str(),
                  is_arg ? "argument" : "result", is_arg ? i : i - n_args,
                  (unsigned long long)b.length, (unsigned long long)desc_bytes(d));
    table.push_back(b);
  }
  for (hxb_hal_buffer_t* t : f->transients)
    table.push_back(hxb_hal_buffer_binding_t{t, 0, hxb_hal_buffer_byte_length(t)});
  const hxb_hal_buffer_binding_table_t tb{(uint32_t)table.size(), table.data()};
  return hxb_hal_device_queue_execute(module->device, wait_semaphore, wait_value, f->cb, &tb,
                                      signal_semaphore, signal_value);
}
