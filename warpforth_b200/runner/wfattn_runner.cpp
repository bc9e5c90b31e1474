// wfattn-runner -- command-line launcher with the interface of WarpForth's
// warpforth-runner (tools/warpforth-runner/warpforth-runner.cpp:7-10,212-253):
//
//   wfattn-runner [kernel.ptx] --kernel NAME --param TYPE:VALUES ... \
//       --grid X,Y,Z --block X,Y,Z --output-param N --output-count N [--impl auto|wfattn|ptx]
//
// TYPE is i64, f64, i64[] or f64[]; array values are comma separated.  The
// output parameter is copied back after the launch and printed as one CSV
// line (17 significant digits for f64).
//
// Launch paths:
//   wfattn  `--kernel attention` with the parameter list of demo/attention.forth
//           (Q, K, V, O arrays, then SEQ_LEN and HEAD_DIM as i64) runs
//           wfattn_attention() from libwfattn.  i64[] arrays carry f32 values
//           packed two per element (the layout the reference's f32 kernel and
//           its tests use, gpu_test/test_kernels.py:805-818); f64[] arrays (the
//           f64 test twin of the kernel) are converted to f32 for the launch and
//           the output back to f64.  No PTX file is needed.
//   ptx     any other kernel: the PTX file is loaded with the CUDA driver API
//           and launched with the given geometry, as the reference runner does.
//           libcuda is opened only on this path.
//   auto    (default) wfattn for `attention`, ptx otherwise.
//
// Errors print a message to stderr and exit with status 1, like the
// reference; library failures print the libwfattn status and message.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <cerrno>
#include <fstream>
#include <sstream>
#include <string>
#include <vector>

#include "wfattn.h"

namespace {

enum class Kind { I64, F64, I64Array, F64Array };

struct Param {
  Kind kind;
  std::vector<int64_t> ints;
  std::vector<double> reals;
  bool is_array() const { return kind == Kind::I64Array || kind == Kind::F64Array; }
  size_t bytes() const { return kind == Kind::I64Array ? ints.size() * 8 : reals.size() * 8; }
};

struct Geometry {
  unsigned x = 1, y = 1, z = 1;
};

[[noreturn]] void die(const std::string &msg) {
  fprintf(stderr, "Error: %s\n", msg.c_str());
  exit(1);
}

void check_cuda(cudaError_t err, const char *what) {
  if (err != cudaSuccess) {
    fprintf(stderr, "CUDA error in %s: %s\n", what, cudaGetErrorString(err));
    exit(1);
  }
}

std::vector<std::string> split(const std::string &s, char sep) {
  std::vector<std::string> out;
  std::string cur;
  for (char c : s) {
    if (c == sep) {
      out.push_back(cur);
      cur.clear();
    } else {
      cur.push_back(c);
    }
  }
  out.push_back(cur);
  return out;
}

int64_t to_i64(const std::string &tok, const std::string &ctx) {
  if (tok.empty()) die("empty integer in " + ctx);
  errno = 0;
  char *end = nullptr;
  long long v = strtoll(tok.c_str(), &end, 10);
  if (errno || *end) die("'" + tok + "' is not an integer (in " + ctx + ")");
  return v;
}

double to_f64(const std::string &tok, const std::string &ctx) {
  if (tok.empty()) die("empty number in " + ctx);
  errno = 0;
  char *end = nullptr;
  double v = strtod(tok.c_str(), &end);
  if (errno == EINVAL || *end) die("'" + tok + "' is not a number (in " + ctx + ")");
  return v;
}

unsigned to_dim(const std::string &tok, const std::string &ctx) {
  const int64_t v = to_i64(tok, ctx);
  if (v < 1 || v > 0x7fffffff) die("dimension out of range in " + ctx);
  return (unsigned)v;
}

Geometry parse_geometry(const std::string &s, const char *opt) {
  const auto parts = split(s, ',');
  if (parts.size() != 3) die(std::string(opt) + " expects X,Y,Z, got: " + s);
  const std::string ctx = std::string(opt) + " " + s;
  return Geometry{to_dim(parts[0], ctx), to_dim(parts[1], ctx), to_dim(parts[2], ctx)};
}

Param parse_param(const std::string &s) {
  const size_t colon = s.find(':');
  if (colon == std::string::npos)
    die("--param needs TYPE:VALUE (i64, f64, i64[] or f64[]), got: " + s);
  const std::string type = s.substr(0, colon), vals = s.substr(colon + 1);
  if (vals.empty()) die("--param has no value: " + s);
  Param p;
  if (type == "i64[]" || type == "f64[]") {
    p.kind = type == "i64[]" ? Kind::I64Array : Kind::F64Array;
    for (const auto &tok : split(vals, ',')) {
      if (p.kind == Kind::I64Array)
        p.ints.push_back(to_i64(tok, "--param " + s));
      else
        p.reals.push_back(to_f64(tok, "--param " + s));
    }
    return p;
  }
  if (vals.find(',') != std::string::npos) die("a scalar --param takes one value: " + s);
  if (type == "i64") {
    p.kind = Kind::I64;
    p.ints.push_back(to_i64(vals, "--param " + s));
  } else if (type == "f64") {
    p.kind = Kind::F64;
    p.reals.push_back(to_f64(vals, "--param " + s));
  } else {
    die("unsupported --param type '" + type + "' (use i64, f64, i64[] or f64[])");
  }
  return p;
}

void print_output(const Param &p, long count) {
  const size_t n = count < 0 ? (p.kind == Kind::I64Array ? p.ints.size() : p.reals.size())
                             : (size_t)count;
  std::string line;
  char buf[64];
  for (size_t i = 0; i < n; ++i) {
    if (i) line.push_back(',');
    if (p.kind == Kind::I64Array) {
      snprintf(buf, sizeof(buf), "%lld", (long long)(i < p.ints.size() ? p.ints[i] : 0));
    } else {
      snprintf(buf, sizeof(buf), "%.17g", i < p.reals.size() ? p.reals[i] : 0.0);
    }
    line += buf;
  }
  printf("%s\n", line.c_str());
}

// ---------------------------------------------------------------- wfattn path
void run_wfattn(std::vector<Param> &params, const Geometry &grid, const Geometry &block,
                bool grid_given, bool block_given, int out_idx) {
  if (params.size() != 6 || !params[0].is_array() || !params[1].is_array() ||
      !params[2].is_array() || !params[3].is_array() || params[4].kind != Kind::I64 ||
      params[5].kind != Kind::I64)
    die("kernel 'attention' takes Q K V O arrays then SEQ_LEN HEAD_DIM as i64 "
        "(demo/attention.forth)");
  const Kind ak = params[0].kind;
  for (int i = 1; i < 4; ++i)
    if (params[i].kind != ak) die("Q, K, V and O must all be i64[] or all f64[]");
  const int64_t S = params[4].ints[0], D = params[5].ints[0];
  if (S < 1 || D < 1) die("SEQ_LEN and HEAD_DIM must be >= 1");
  const size_t n = (size_t)S * (size_t)D;
  // Host f32 copies of the four arrays (zero padded to S*D).
  std::vector<std::vector<float>> host(4, std::vector<float>(n, 0.f));
  for (int i = 0; i < 4; ++i) {
    const Param &p = params[i];
    if (ak == Kind::I64Array) {
      const size_t avail = p.ints.size() * 2;
      std::vector<float> tmp(avail);
      memcpy(tmp.data(), p.ints.data(), p.ints.size() * 8);
      for (size_t j = 0; j < n && j < avail; ++j) host[i][j] = tmp[j];
    } else {
      for (size_t j = 0; j < n && j < p.reals.size(); ++j) host[i][j] = (float)p.reals[j];
    }
  }
  float *dev[4] = {nullptr, nullptr, nullptr, nullptr};
  for (int i = 0; i < 4; ++i) {
    check_cuda(cudaMalloc(&dev[i], n * sizeof(float)), "cudaMalloc");
    check_cuda(cudaMemcpy(dev[i], host[i].data(), n * sizeof(float), cudaMemcpyHostToDevice),
               "cudaMemcpy H2D");
  }
  wfattn_dim3 g{grid.x, grid.y, grid.z}, b{block.x, block.y, block.z};
  wfattn_status_t st = wfattn_attention(dev[0], dev[1], dev[2], dev[3], S, D,
                                        grid_given ? &g : nullptr, block_given ? &b : nullptr,
                                        nullptr);
  if (st != WFATTN_OK) {
    fprintf(stderr, "wfattn error: %s: %s\n", wfattn_status_string(st), wfattn_last_error());
    exit(1);
  }
  check_cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
  st = wfattn_device_status(nullptr, 1);
  if (st != WFATTN_OK) {
    fprintf(stderr, "wfattn error: %s: %s\n", wfattn_status_string(st), wfattn_last_error());
    exit(1);
  }
  for (int i = 0; i < 4; ++i) {
    check_cuda(cudaMemcpy(host[i].data(), dev[i], n * sizeof(float), cudaMemcpyDeviceToHost),
               "cudaMemcpy D2H");
    cudaFree(dev[i]);
  }
  // Write every array back into its parameter so --output-param can select any of them.
  for (int i = 0; i < 4; ++i) {
    Param &p = params[i];
    if (ak == Kind::I64Array) {
      const size_t nbytes = p.ints.size() * 8;
      std::vector<uint8_t> raw(nbytes, 0);
      memcpy(raw.data(), host[i].data(), std::min(nbytes, n * sizeof(float)));
      if (n * sizeof(float) < nbytes) {
        // keep the caller's trailing bytes beyond S*D floats
        memcpy(raw.data() + n * sizeof(float),
               reinterpret_cast<uint8_t *>(p.ints.data()) + n * sizeof(float),
               nbytes - n * sizeof(float));
      }
      memcpy(p.ints.data(), raw.data(), nbytes);
    } else {
      for (size_t j = 0; j < n && j < p.reals.size(); ++j) p.reals[j] = host[i][j];
    }
  }
  (void)out_idx;
}

// ---------------------------------------------------------------- PTX path
typedef int CUres;
typedef int CUdev;
typedef void *CUctx;
typedef void *CUmod;
typedef void *CUfn;
typedef unsigned long long CUptr;

struct Driver {
  void *h = nullptr;
  CUres (*Init)(unsigned);
  CUres (*DeviceGet)(CUdev *, int);
  CUres (*CtxCreate)(CUctx *, unsigned, CUdev);
  CUres (*ModuleLoadData)(CUmod *, const void *);
  CUres (*ModuleGetFunction)(CUfn *, CUmod, const char *);
  CUres (*MemAlloc)(CUptr *, size_t);
  CUres (*MemcpyHtoD)(CUptr, const void *, size_t);
  CUres (*MemcpyDtoH)(void *, CUptr, size_t);
  CUres (*LaunchKernel)(CUfn, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned,
                        unsigned, void *, void **, void **);
  CUres (*CtxSynchronize)();
  CUres (*MemFree)(CUptr);
  CUres (*GetErrorString)(CUres, const char **);
};

template <typename F>
void bind(Driver &d, F &fn, const char *name) {
  fn = reinterpret_cast<F>(dlsym(d.h, name));
  if (!fn) die(std::string("libcuda has no ") + name);
}

void check_cu(const Driver &d, CUres r, const char *what) {
  if (r != 0) {
    const char *s = nullptr;
    d.GetErrorString(r, &s);
    fprintf(stderr, "CUDA error in %s: %s\n", what, s ? s : "unknown");
    exit(1);
  }
}

void run_ptx(const std::string &ptx_file, const std::string &kernel, std::vector<Param> &params,
             const Geometry &grid, const Geometry &block) {
  std::ifstream f(ptx_file, std::ios::binary);
  if (!f) die("cannot open " + ptx_file);
  std::stringstream ss;
  ss << f.rdbuf();
  const std::string ptx = ss.str();
  Driver d;
  d.h = dlopen("libcuda.so.1", RTLD_NOW);
  if (!d.h) die("the PTX path needs the CUDA driver (libcuda.so.1)");
  bind(d, d.Init, "cuInit");
  bind(d, d.DeviceGet, "cuDeviceGet");
  bind(d, d.CtxCreate, "cuCtxCreate_v2");
  bind(d, d.ModuleLoadData, "cuModuleLoadData");
  bind(d, d.ModuleGetFunction, "cuModuleGetFunction");
  bind(d, d.MemAlloc, "cuMemAlloc_v2");
  bind(d, d.MemcpyHtoD, "cuMemcpyHtoD_v2");
  bind(d, d.MemcpyDtoH, "cuMemcpyDtoH_v2");
  bind(d, d.LaunchKernel, "cuLaunchKernel");
  bind(d, d.CtxSynchronize, "cuCtxSynchronize");
  bind(d, d.MemFree, "cuMemFree_v2");
  bind(d, d.GetErrorString, "cuGetErrorString");
  check_cu(d, d.Init(0), "cuInit");
  CUdev dev;
  check_cu(d, d.DeviceGet(&dev, 0), "cuDeviceGet");
  CUctx ctx;
  check_cu(d, d.CtxCreate(&ctx, 0, dev), "cuCtxCreate");
  CUmod mod;
  check_cu(d, d.ModuleLoadData(&mod, ptx.c_str()), "cuModuleLoadData");
  CUfn fn;
  check_cu(d, d.ModuleGetFunction(&fn, mod, kernel.c_str()), "cuModuleGetFunction");
  std::vector<CUptr> ptrs(params.size(), 0);
  std::vector<void *> args(params.size());
  for (size_t i = 0; i < params.size(); ++i) {
    Param &p = params[i];
    if (p.is_array()) {
      const void *src = p.kind == Kind::I64Array ? (const void *)p.ints.data()
                                                 : (const void *)p.reals.data();
      check_cu(d, d.MemAlloc(&ptrs[i], p.bytes()), "cuMemAlloc");
      check_cu(d, d.MemcpyHtoD(ptrs[i], src, p.bytes()), "cuMemcpyHtoD");
      args[i] = &ptrs[i];
    } else {
      args[i] = p.kind == Kind::I64 ? (void *)p.ints.data() : (void *)p.reals.data();
    }
  }
  check_cu(d, d.LaunchKernel(fn, grid.x, grid.y, grid.z, block.x, block.y, block.z, 0, nullptr,
                             args.data(), nullptr),
           "cuLaunchKernel");
  check_cu(d, d.CtxSynchronize(), "cuCtxSynchronize");
  for (size_t i = 0; i < params.size(); ++i) {
    Param &p = params[i];
    if (!p.is_array()) continue;
    void *dst = p.kind == Kind::I64Array ? (void *)p.ints.data() : (void *)p.reals.data();
    check_cu(d, d.MemcpyDtoH(dst, ptrs[i], p.bytes()), "cuMemcpyDtoH");
    d.MemFree(ptrs[i]);
  }
}

const char *kUsage =
    "Usage: wfattn-runner [kernel.ptx] --kernel NAME [--param i64[]:V,...] [--param f64[]:V,...] "
    "[--param i64:V] [--param f64:V] [--grid X,Y,Z] [--block X,Y,Z] [--output-param N] "
    "[--output-count N] [--impl auto|wfattn|ptx]\n";

}  // namespace

int main(int argc, char **argv) {
  std::string ptx_file, kernel, impl = "auto";
  std::vector<Param> params;
  Geometry grid, block;
  bool grid_given = false, block_given = false;
  long out_idx = 0, out_count = -1;
  for (int i = 1; i < argc; ++i) {
    const std::string a = argv[i];
    auto value = [&]() -> std::string {
      if (i + 1 >= argc) die(a + " requires a value");
      return argv[++i];
    };
    if (a == "--param") {
      params.push_back(parse_param(value()));
    } else if (a == "--grid") {
      grid = parse_geometry(value(), "--grid");
      grid_given = true;
    } else if (a == "--block") {
      block = parse_geometry(value(), "--block");
      block_given = true;
    } else if (a == "--output-param") {
      out_idx = (long)to_i64(value(), "--output-param");
    } else if (a == "--output-count") {
      out_count = (long)to_i64(value(), "--output-count");
    } else if (a == "--kernel") {
      kernel = value();
    } else if (a == "--impl") {
      impl = value();
      if (impl != "auto" && impl != "wfattn" && impl != "ptx")
        die("--impl must be auto, wfattn or ptx");
    } else if (!a.empty() && a[0] == '-') {
      die("unknown option " + a);
    } else {
      ptx_file = a;
    }
  }
  if (kernel.empty()) {
    fputs(kUsage, stderr);
    die("--kernel NAME is required");
  }
  if (params.empty()) die("at least one --param is required");
  if (out_idx < 0 || out_idx >= (long)params.size())
    die("output-param " + std::to_string(out_idx) + " out of range (have " +
        std::to_string(params.size()) + " params)");
  if (!params[out_idx].is_array())
    die("output-param " + std::to_string(out_idx) + " is a scalar (cannot read back)");
  const bool use_wfattn = impl == "wfattn" || (impl == "auto" && kernel == "attention");
  if (use_wfattn) {
    if (kernel != "attention") die("libwfattn implements kernel 'attention' only");
    run_wfattn(params, grid, block, grid_given, block_given, (int)out_idx);
  } else {
    if (ptx_file.empty()) {
      fputs(kUsage, stderr);
      die("a PTX file is required for kernel '" + kernel + "'");
    }
    run_ptx(ptx_file, kernel, params, grid, block);
  }
  print_output(params[out_idx], out_count);
  return 0;
}
