"""Compile the reference's own LIF-FDE kernel sources for the host CPU (oracle/_ref/).

TEST INFRASTRUCTURE ONLY.  The reference (cjge-ustc/DF-SNN-official) ships its kernels as
CUDA C strings inside Python modules (spikeDE_dis/fde_cupy_kernels_all.py,
examples/cnn128/aligned_glmulti.py, spikeDE_dis/direct_euler_cupy.py).  This recipe reads
those strings from the reference checkout, where they lie, wraps them with
oracle/ref_shim.h (a host-side stand-in for the CUDA thread indices) and compiles them with
g++ into oracle/_ref/libdfsnn_ref.so.  Nothing of the reference is committed: the generated
sources and the library live only under oracle/_ref/ (git-ignored).

Floating-point contraction follows the reference's compile flags: the library kernels are
built by NVRTC with its default --fmad=true (here: -ffp-contract=fast with FMA hardware),
the aligned kernels with --fmad=false (here: -ffp-contract=off).

The same kernel source texts are also compiled for the GPU (build_cuda): every text the
reference hands to cupy.RawKernel, with the options it passes (none for
spikeDE_dis/fde_cupy_kernels_all.py and direct_euler_cupy.py; --fmad=false for the
examples' aligned kernels, with HISTORY_RHO substituted into the text as the reference
does), one nvcc cubin per text for sm_100 (the target CuPy's NVRTC build uses on a B200),
into oracle/_ref/cuda/ with a manifest keyed by source and options.  oracle/cupy_standin
launches them, so that the reference's own Python code runs its own kernels on the GPU.

The reference checkout is found at $DFSNN_REFERENCE, else at DEFAULT_REFERENCE.

Usage: python oracle/build_ref.py [--reference PATH] [--no-cuda]
Exits 0 without building when the reference checkout is absent.
"""
import argparse
import ast
import os
import subprocess
import sys
import types

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
CUDA_OUT = os.path.join(OUT, "cuda")
DEFAULT_REFERENCE = "/root/reference"
# The examples' HISTORY_RHO values prebuilt for the GPU: 1.0 is the value every shipped
# policy uses (examples/cnn128/train_ablation.py:21); 0.5 lets tests exercise the rho path.
ALIGNED_RHOS = (1.0, 0.5)
CUDA_ARCH = ["-gencode", "arch=compute_100,code=sm_100"]


def reference_path(explicit=None):
    return explicit or os.environ.get("DFSNN_REFERENCE") or DEFAULT_REFERENCE


# The reference's kernels that run one thread per neuron with no inter-thread traffic.
LIB_KERNELS = [
    "gl_forward_kernel_code", "gl_backward_kernel_code",
    "gl1_forward_kernel_code", "gl1_backward_kernel_code",
    "trap_forward_kernel_code", "trap_backward_kernel_code",
    "predictor_forward_kernel_code", "predictor_backward_kernel_code",
    "vo_gl1_forward_kernel_code",
    "glmulti_backward_kernel_code", "glmulti_full_backward_kernel_code",
    "trap1_forward_kernel_code", "trap1_backward_kernel_code",
    "predictor1_forward_kernel_code", "predictor1_backward_kernel_code",
    "euler_forward_kernel_code", "euler_backward_kernel_code",
    "vo_gl1_backward_kernel_code", "vo_gl1_full_backward_kernel_code",
    "fa_gl1_forward_kernel_code", "fa_gl1_backward_kernel_code", "fa_gl1_full_backward_kernel_code",
    "vo_predictor_forward_kernel_code", "vo_predictor_backward_kernel_code",
]

# Statements whose fused multiply-add NVRTC forms but GCC does not (see collect_sources).
NVRTC_CONTRACTIONS = [
    ("hist += trap_weights[weight_idx] * v_seq_local[hist_idx];",
     "hist = fmaf(trap_weights[weight_idx], v_seq_local[hist_idx], hist);"),
    ("grad_v_mem -= c_rev[weight_idx] * grad_v;",
     "grad_v_mem = fmaf(-c_rev[weight_idx], grad_v, grad_v_mem);"),
    ("grad_v_mem -= trap_weights[weight_idx] * grad_v;",
     "grad_v_mem = fmaf(-trap_weights[weight_idx], grad_v, grad_v_mem);"),
    ("hist_integral += predictor_weights[weight_idx] * hist_dv;",
     "hist_integral = fmaf(predictor_weights[weight_idx], hist_dv, hist_integral);"),
    ("hist += weights[wi] * drift_seq[i * N + n];",
     "hist = fmaf(weights[wi], drift_seq[i * N + n], hist);"),
    ("hist += weights[wi] * v_hist_seq[i * N + n];",
     "hist = fmaf(weights[wi], v_hist_seq[i * N + n], hist);"),
    ("grad_hist[i] -= weights[wi] * grad_pre;",
     "grad_hist[i] = fmaf(-weights[wi], grad_pre, grad_hist[i]);"),
]

# Host launchers (this repository's code): one OpenMP loop over global thread indices.
WRAPPERS_FMA = r'''
#define DFSNN_REF_LOOP(NTHREADS, CALL)                                   \
    do {                                                                  \
        const long long _total = ((long long)(NTHREADS) + 255) / 256 * 256; \
        _Pragma("omp parallel for schedule(static)")                      \
        for (long long _g = 0; _g < _total; ++_g) {                       \
            dfsnn_ref_set_thread(_g);                                     \
            CALL;                                                         \
        }                                                                 \
    } while (0)

extern "C" {
void ref_gl_forward(const float* x, const float* v0, const float* w, float* s, float* v,
                    int T, int N, float tau, float beta, float th, float v_reset) {
    DFSNN_REF_LOOP(N, lif_fde_gl_forward_kernel(x, v0, w, s, v, T, N, tau, beta, th, v_reset));
}
void ref_gl_backward(const float* gs, const float* gv, const float* x, const float* v0,
                     const float* w, float* gx, float* gv0, int T, int N, float tau, float beta,
                     float th, float sg) {
    DFSNN_REF_LOOP(N, lif_fde_gl_backward_kernel(gs, gv, x, v0, w, gx, gv0, T, N, tau, beta, th, sg));
}
void ref_gl1_forward(const float* x, const float* v0, const float* w, float* s, float* v,
                     int T, int N, float tau, float beta, float th, float v_reset, float h_beta) {
    DFSNN_REF_LOOP(N, lif_fde_gl1_forward_kernel(x, v0, w, s, v, T, N, tau, beta, th, v_reset, h_beta));
}
void ref_gl1_backward(const float* gs, const float* gv, const float* x, const float* v0,
                      const float* w, float* gx, float* gv0, int T, int N, float tau, float beta,
                      float th, float sg, float h_beta) {
    DFSNN_REF_LOOP(N, lif_fde_gl1_backward_kernel(gs, gv, x, v0, w, gx, gv0, T, N, tau, beta, th, sg, h_beta));
}
void ref_trap_forward(const float* x, const float* v0, const float* w, float* s, float* v,
                      int T, int N, float tau, float beta, float th, float v_reset) {
    DFSNN_REF_LOOP(N, lif_fde_trap_forward_kernel(x, v0, w, s, v, T, N, tau, beta, th, v_reset));
}
void ref_trap_backward(const float* gs, const float* gv, const float* x, const float* v0,
                       const float* w, float* gx, float* gv0, int T, int N, float tau, float beta,
                       float th, float sg) {
    DFSNN_REF_LOOP(N, lif_fde_trap_backward_kernel(gs, gv, x, v0, w, gx, gv0, T, N, tau, beta, th, sg));
}
void ref_predictor_forward(const float* x, const float* v0, const float* w, float* s, float* v,
                           int T, int N, float tau, float beta, float th, float v_reset,
                           float h_beta, float gamma1) {
    DFSNN_REF_LOOP(N, lif_fde_predictor_forward_kernel(x, v0, w, s, v, T, N, tau, beta, th, v_reset, h_beta, gamma1));
}
void ref_predictor_backward(const float* gs, const float* gv, const float* x, const float* v0,
                            const float* w, float* gx, float* gv0, int T, int N, float tau,
                            float beta, float th, float sg, float h_beta, float gamma1) {
    DFSNN_REF_LOOP(N, lif_fde_predictor_backward_kernel(gs, gv, x, v0, w, gx, gv0, T, N, tau, beta, th, sg, h_beta, gamma1));
}
void ref_trap1_forward(const float* x, const float* v0, const float* w, float* s, float* v,
                       int T, int N, float tau, float beta, float th, float v_reset, float h_beta) {
    DFSNN_REF_LOOP(N, lif_fde_trap1_forward_kernel(x, v0, w, s, v, T, N, tau, beta, th, v_reset, h_beta));
}
void ref_trap1_backward(const float* gs, const float* gv, const float* x, const float* v0,
                        const float* w, float* gx, float* gv0, int T, int N, float tau, float beta,
                        float th, float sg, float h_beta) {
    DFSNN_REF_LOOP(N, lif_fde_trap1_backward_kernel(gs, gv, x, v0, w, gx, gv0, T, N, tau, beta, th, sg, h_beta));
}
void ref_predictor1_forward(const float* x, const float* v0, const float* w, float* s, float* v,
                            int T, int N, float tau, float beta, float th, float v_reset,
                            float h_beta, float gamma1) {
    DFSNN_REF_LOOP(N, lif_fde_predictor1_forward_kernel(x, v0, w, s, v, T, N, tau, beta, th, v_reset, h_beta, gamma1));
}
void ref_predictor1_backward(const float* gs, const float* gv, const float* x, const float* v0,
                             const float* w, float* gx, float* gv0, int T, int N, float tau,
                             float beta, float th, float sg, float h_beta, float gamma1) {
    DFSNN_REF_LOOP(N, lif_fde_predictor1_backward_kernel(gs, gv, x, v0, w, gx, gv0, T, N, tau, beta, th, sg, h_beta, gamma1));
}
void ref_lifeuler_forward(const float* x, const float* v0, float* s, float* v, int T, int N,
                          float tau, float th, float v_reset) {
    DFSNN_REF_LOOP(N, lif_euler_forward_kernel(x, v0, s, v, T, N, tau, th, v_reset));
}
void ref_lifeuler_backward(const float* gs, const float* gv, const float* x, const float* v0,
                           float* gx, float* gv0, int T, int N, float tau, float th, float sg) {
    DFSNN_REF_LOOP(N, lif_euler_backward_kernel(gs, gv, x, v0, gx, gv0, T, N, tau, th, sg));
}
void ref_vogl1_forward(const float* x, const float* v0, const float* scale, const float* W,
                       float* s, float* vpre, float* vhist, float* drift, int T, int N, int B,
                       int per_batch, float tau, float th) {
    DFSNN_REF_LOOP(N, lif_fde_vo_gl1_forward_kernel(x, v0, scale, W, s, vpre, vhist, drift, T, N, B, per_batch, tau, th));
}
void ref_vogl1_backward(int full, const float* gs, const float* scale, const float* W,
                        const float* vpre, float* gx, float* gv0, float* gpre, int T, int N,
                        int B, int per_batch, float tau, float th, float sg) {
    if (full)
        DFSNN_REF_LOOP(N, lif_fde_vo_gl1_full_backward_kernel(gs, scale, W, vpre, gx, gv0, gpre, T, N, B, per_batch, tau, th, sg));
    else
        DFSNN_REF_LOOP(N, lif_fde_vo_gl1_backward_kernel(gs, scale, W, vpre, gx, gv0, gpre, T, N, B, per_batch, tau, th, sg));
}
void ref_fagl1_forward(const float* x, const float* v0, const float* W, float* s, float* vpre,
                       float* vhist, int T, int N, int B, int per_batch, float tau, float hb,
                       float th) {
    DFSNN_REF_LOOP(N, lif_fde_fa_gl1_forward_kernel(x, v0, W, s, vpre, vhist, T, N, B, per_batch, tau, hb, th));
}
void ref_fagl1_backward(int full, const float* gs, const float* W, const float* vpre, float* gx,
                        float* gv0, float* gpre, int T, int N, int B, int per_batch, float tau,
                        float hb, float th, float sg) {
    if (full)
        DFSNN_REF_LOOP(N, lif_fde_fa_gl1_full_backward_kernel(gs, W, vpre, gx, gv0, gpre, T, N, B, per_batch, tau, hb, th, sg));
    else
        DFSNN_REF_LOOP(N, lif_fde_fa_gl1_backward_kernel(gs, W, vpre, gx, gv0, gpre, T, N, B, per_batch, tau, hb, th, sg));
}
void ref_vopred_forward(const float* x, const float* v0, const float* scale, const float* W,
                        float* s, float* vpre, float* drift, int T, int N, int B, int per_batch,
                        float tau, float th, float rm) {
    DFSNN_REF_LOOP(N, lif_fde_vo_predictor_forward_kernel(x, v0, scale, W, s, vpre, drift, T, N, B, per_batch, tau, th, rm));
}
void ref_vopred_backward(const float* gs, const float* scale, const float* W, const float* vpre,
                         float* gx, float* gv0, float* gpre, int T, int N, int B, int per_batch,
                         float tau, float th, float sg, float rm) {
    DFSNN_REF_LOOP(N, lif_fde_vo_predictor_backward_kernel(gs, scale, W, vpre, gx, gv0, gpre, T, N, B, per_batch, tau, th, sg, rm));
}
void ref_weighted_sum_f32(const float* coeff, const float* history, float* out, int L, int S) {
    DFSNN_REF_LOOP(S, weighted_sum_f32(coeff, history, out, L, S));
}
void ref_weighted_sum_f64(const double* coeff, const double* history, double* out, int L, int S) {
    DFSNN_REF_LOOP(S, weighted_sum_f64(coeff, history, out, L, S));
}
void ref_glmulti_forward(const float* x, const float* v0, const float* scale, const float* W,
                         float* s, float* vpre, float* vhist, float* drift, int T, int N,
                         float tau, float th) {
    DFSNN_REF_LOOP(N, lif_fde_vo_gl1_forward_kernel(x, v0, scale, W, s, vpre, vhist, drift, T, N, 1, 0, tau, th));
}
void ref_glmulti_backward(int full, const float* gs, const float* scale, const float* W,
                          const float* vpre, float* gx, float* gv0, float* gpre, int T, int N,
                          float tau, float th, float sg) {
    if (full)
        DFSNN_REF_LOOP(N, lif_fde_glmulti_full_backward_kernel(gs, scale, W, vpre, gx, gv0, gpre, T, N, tau, th, sg));
    else
        DFSNN_REF_LOOP(N, lif_fde_glmulti_backward_kernel(gs, scale, vpre, gx, gv0, gpre, T, N, tau, th, sg));
}
void ref_euler_forward(const float* x, const float* z0, float* s, float* zpre, float* sin_,
                       float* zf, int T, int N, float in_scale, float gain, float bias, float tau,
                       float th, float step, float reset_strength, float sdt) {
    DFSNN_REF_LOOP(N, direct_lif_euler_forward(x, z0, s, zpre, sin_, zf, T, N, in_scale, gain, bias, tau, th, step, reset_strength, sdt));
}
void ref_euler_backward(const float* gs, const float* gzf, const float* x, const float* zpre,
                        const float* sin_, float* gx, float* gz0, float* g_scale, float* g_gain,
                        float* g_bias, int T, int N, float in_scale, float gain, float tau,
                        float step, float sg, float sdt) {
    DFSNN_REF_LOOP(N, direct_lif_euler_backward(gs, gzf, x, zpre, sin_, gx, gz0, g_scale, g_gain, g_bias, T, N, in_scale, gain, tau, step, sg, sdt));
}
}
'''

WRAPPERS_NOFMA = r'''
extern "C" {
void ref_aligned_forward(const float* x, const float* v0, const float* a, const float* w,
                         float* s, float* p, float* hist, int T, int N, float tau, float th) {
    const long long total = ((long long)N + 255) / 256 * 256;
#pragma omp parallel for schedule(static)
    for (long long g = 0; g < total; ++g) {
        dfsnn_ref_set_thread(g);
        aligned_forward(x, v0, a, w, s, p, hist, T, N, tau, th);
    }
}
void ref_aligned_backward(const float* g, const float* a, const float* w, const float* p,
                          float* gx, float* gv, float* ga, int T, int N, float tau, float th,
                          float sg, float rho) {
    dfsnn_ref_rho = rho;
    const long long total = ((long long)N + 255) / 256 * 256;
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < total; ++i) {
        dfsnn_ref_set_thread(i);
        aligned_backward(g, a, w, p, gx, gv, ga, T, N, tau, th, sg);
    }
}
}
'''


def _stub_h5py():
    # spikeDE_dis/__init__ imports solver.py, which imports h5py.h5z.FLAG_SKIP_EDC.
    if "h5py" not in sys.modules:
        h5 = types.ModuleType("h5py")
        h5z = types.ModuleType("h5py.h5z")
        h5z.FLAG_SKIP_EDC = 0
        h5.h5z = h5z
        sys.modules["h5py"] = h5
        sys.modules["h5py.h5z"] = h5z


def _function_local_string(path, func_name, var_name="code"):
    """Return the string literal assigned to `var_name` inside `func_name` of a file."""
    with open(path) as f:
        tree = ast.parse(f.read())
    for node in ast.walk(tree):
        if isinstance(node, ast.FunctionDef) and node.name == func_name:
            for sub in ast.walk(node):
                if (isinstance(sub, ast.Assign) and len(sub.targets) == 1
                        and isinstance(sub.targets[0], ast.Name) and sub.targets[0].id == var_name
                        and isinstance(sub.value, ast.Constant) and isinstance(sub.value.value, str)):
                    return sub.value.value
    raise RuntimeError(f"{func_name}.{var_name} not found in {path}")


def _weighted_sum_sources(path):
    """The weighted_sum kernel of solver.py (_get_weighted_sum_kernel, :77-104) is an f-string
    over the element type; rebuild it for float and double from the file's syntax tree
    (nothing of solver.py is imported), with NVRTC's contraction of the accumulation."""
    with open(path) as f:
        tree = ast.parse(f.read())
    template = None
    for node in ast.walk(tree):
        if isinstance(node, ast.FunctionDef) and node.name == "_get_weighted_sum_kernel":
            for sub in ast.walk(node):
                if (isinstance(sub, ast.Assign) and len(sub.targets) == 1
                        and isinstance(sub.targets[0], ast.Name) and sub.targets[0].id == "code"
                        and isinstance(sub.value, ast.JoinedStr)):
                    template = sub.value
    if template is None:
        raise RuntimeError("_get_weighted_sum_kernel.code not found in " + path)
    out = []
    for type_name, suffix, fma in (("float", "f32", "fmaf"), ("double", "f64", "fma")):
        text = ""
        for part in template.values:
            if isinstance(part, ast.Constant):
                text += part.value
            elif isinstance(part, ast.FormattedValue) and isinstance(part.value, ast.Name) \
                    and part.value.id == "type_name":
                text += type_name
            else:
                raise RuntimeError("unexpected field in the weighted_sum template")
        stmt = "acc += coeff[j] * history[j * state_size + idx];"
        if stmt not in text or "void weighted_sum(" not in text:
            raise RuntimeError("weighted_sum kernel body not recognised")
        text = text.replace(stmt, f"acc = {fma}(coeff[j], history[j * state_size + idx], acc);")
        out.append(text.replace("void weighted_sum(", f"void weighted_sum_{suffix}("))
    return "\n".join(out)


def collect_sources(reference):
    _stub_h5py()
    sys.path.insert(0, reference)
    sys.path.insert(0, os.path.join(reference, "examples", "cnn128"))
    import spikeDE_dis.fde_cupy_kernels_all as lib  # noqa: E402
    import aligned_glmulti as alg  # noqa: E402
    fma_parts = [getattr(lib, name) for name in LIB_KERNELS]
    # NVRTC (--fmad=true) contracts every a += b*c / a -= b*c; GCC's -ffp-contract=fast leaves
    # these loop statements of the GL1 / TRAP1 / PREDICTOR1 backward unfused (found by stepping
    # one neuron through both), so the host build writes NVRTC's contraction out.
    for i, part in enumerate(fma_parts):
        for old, new in NVRTC_CONTRACTIONS:
            part = part.replace(old, new)
        fma_parts[i] = part
    euler_path = os.path.join(reference, "spikeDE_dis", "direct_euler_cupy.py")
    fma_parts.append(_function_local_string(euler_path, "_get_forward_kernel"))
    fma_parts.append(_function_local_string(euler_path, "_get_backward_kernel"))
    fma_parts.append(_weighted_sum_sources(os.path.join(reference, "spikeDE_dis", "solver.py")))
    # The reference substitutes HISTORY_RHO into this statement as text before compiling
    # (aligned_glmulti.py:90); do the same with a run-time variable.
    target = "adj[j]-=w[t*T+j]*r;"
    if target not in alg.BACKWARD:
        raise RuntimeError("aligned_backward history statement not found")
    backward = alg.BACKWARD.replace(target, "adj[j]-=dfsnn_ref_rho*w[t*T+j]*r;")
    nofma = "static float dfsnn_ref_rho = 1.0f;\n" + alg.FORWARD + backward
    return "\n".join(fma_parts), nofma


def build(reference, cxx="g++"):
    if not os.path.isdir(os.path.join(reference, "spikeDE_dis")):
        print(f"build_ref: no reference checkout at {reference}; skipped")
        return None
    os.makedirs(OUT, exist_ok=True)
    fma_src, nofma_src = collect_sources(reference)
    shim = '#include "%s"\n' % os.path.join(HERE, "ref_shim.h")
    fma_cpp = os.path.join(OUT, "ref_kernels_fma.cpp")
    nofma_cpp = os.path.join(OUT, "ref_kernels_nofma.cpp")
    with open(fma_cpp, "w") as f:
        f.write(shim + fma_src + WRAPPERS_FMA)
    with open(nofma_cpp, "w") as f:
        f.write(shim + nofma_src + WRAPPERS_NOFMA)
    common = ["-O2", "-fPIC", "-fopenmp", "-march=x86-64-v3", "-fno-fast-math", "-w"]
    objs = []
    for src, contract in ((fma_cpp, "fast"), (nofma_cpp, "off")):
        obj = src[:-4] + ".o"
        subprocess.check_call([cxx, *common, f"-ffp-contract={contract}", "-c", src, "-o", obj])
        objs.append(obj)
    lib = os.path.join(OUT, "libdfsnn_ref.so")
    subprocess.check_call([cxx, "-shared", "-fopenmp", *objs, "-o", lib])
    print(f"build_ref: built {lib}")
    return lib


def _source_key():
    import importlib.util
    path = os.path.join(HERE, "cupy_standin", "cupy", "_source_key.py")
    spec = importlib.util.spec_from_file_location("dfsnn_ref_source_key", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.source_key


def cuda_sources(reference):
    """(code, options) pairs exactly as the reference passes them to cupy.RawKernel."""
    _stub_h5py()
    for p in (reference, os.path.join(reference, "examples", "cnn128")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import spikeDE_dis.fde_cupy_kernels_all as lib  # noqa: E402
    import aligned_glmulti as alg  # noqa: E402
    out = [(getattr(lib, name), ()) for name in sorted(dir(lib)) if name.endswith("_kernel_code")]
    euler_path = os.path.join(reference, "spikeDE_dis", "direct_euler_cupy.py")
    out.append((_function_local_string(euler_path, "_get_forward_kernel"), ()))
    out.append((_function_local_string(euler_path, "_get_backward_kernel"), ()))
    target = "adj[j]-=w[t*T+j]*r;"
    if target not in alg.BACKWARD:
        raise RuntimeError("aligned_backward history statement not found")
    for rho in ALIGNED_RHOS:
        # the text substitution of examples/cnn128/aligned_glmulti.py:90
        code = alg.BACKWARD.replace(target, f"adj[j]-={rho:.8f}f*w[t*T+j]*r;")
        out.append((alg.FORWARD + code, ("--fmad=false",)))
    return out


_C_SIZES = {"int": 4, "unsigned": 4, "unsigned int": 4, "float": 4, "double": 8,
            "long long": 8, "unsigned long long": 8, "size_t": 8, "bool": 1, "char": 1}


def kernel_params(code, name):
    """Byte size of every parameter of kernel `name` in `code` (8 for pointers), read from
    its declaration, so that a launch can be checked against it before it reaches the GPU."""
    import re
    m = re.search(r"__global__\s+void\s+" + re.escape(name) + r"\s*\(([^)]*)\)", code)
    if not m:
        raise RuntimeError(f"kernel {name}: declaration not found")
    sizes = []
    for decl in m.group(1).split(","):
        decl = decl.strip()
        if not decl:
            continue
        if "*" in decl:
            sizes.append(8)
            continue
        words = [w for w in re.sub(r"\b(const|__restrict__|volatile)\b", " ", decl).split()]
        ctype = " ".join(words[:-1])
        if ctype not in _C_SIZES:
            raise RuntimeError(f"kernel {name}: unknown parameter type '{ctype}'")
        sizes.append(_C_SIZES[ctype])
    return sizes


def build_cuda(reference, nvcc=None):
    import json
    import re
    if not os.path.isdir(os.path.join(reference, "spikeDE_dis")):
        print(f"build_ref: no reference checkout at {reference}; CUDA build skipped")
        return None
    nvcc = nvcc or os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    key_of = _source_key()
    os.makedirs(CUDA_OUT, exist_ok=True)
    manifest, procs = {}, []
    for code, options in cuda_sources(reference):
        key = key_of(code, options)
        if key in manifest:
            continue
        names = re.findall(r"__global__\s+void\s+(\w+)", code)
        src = os.path.join(CUDA_OUT, key + ".cu")
        cubin = os.path.join(CUDA_OUT, key + ".cubin")
        with open(src, "w") as f:
            f.write(code)
        manifest[key] = {"cubin": key + ".cubin", "names": names, "options": list(options),
                         "params": {n: kernel_params(code, n) for n in names}}
        procs.append(subprocess.Popen([nvcc, "-cubin", *CUDA_ARCH, *options, "-w", src,
                                       "-o", cubin]))
    if any(p.wait() != 0 for p in procs):
        raise RuntimeError("build_ref: nvcc failed on a reference kernel source")
    with open(os.path.join(CUDA_OUT, "manifest.json"), "w") as f:
        json.dump(manifest, f, indent=1)
    print(f"build_ref: built {len(manifest)} reference kernel modules for sm_100 in {CUDA_OUT}")
    return CUDA_OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=None)
    ap.add_argument("--cxx", default="g++")
    ap.add_argument("--no-cuda", action="store_true")
    args = ap.parse_args()
    ref = reference_path(args.reference)
    build(ref, args.cxx)
    if not args.no_cuda:
        build_cuda(ref)
