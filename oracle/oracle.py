"""numpy front end of the LIF-FDE oracle (TEST INFRASTRUCTURE ONLY).

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference legs import
this module, as the checker or as the timed CPU baseline.  It loads
  * oracle/build/liboracle.so     -- the C restatement (oracle/lif_fde_oracle.c), and
  * oracle/_ref/libdfsnn_ref.so   -- the reference's own kernel sources compiled for the
                                     host by oracle/build_ref.py, when it was built.
Arrays are time-major [T, N] float32, as the reference's autograd Functions pass them.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "build", "liboracle.so")
REF_PATH = os.path.join(HERE, "_ref", "libdfsnn_ref.so")

GL, TRAP, PRED, GL1, TRAP1, PRED1, EULER = 0, 1, 2, 3, 4, 5, 6
SCHEMES = {"gl": GL, "trap": TRAP, "predictor": PRED, "gl1": GL1, "trap1": TRAP1,
           "predictor1": PRED1, "euler": EULER}
RECOMPUTE_BACKWARD = ("trap1", "predictor1")   # backward recomputes with a plain sum

_f = ctypes.c_float
_i = ctypes.c_int
_i64 = ctypes.c_int64
_p = ctypes.c_void_p

_lib = None
_ref = None


def build():
    """Compile the C restatement (make -C oracle)."""
    subprocess.check_call(["make", "-s", "-C", HERE])


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        L.orc_single_forward.argtypes = [_i, _p, _p, _p, _p, _p, _i, _i64, _f, _f, _f, _f, _f]
        L.orc_single_backward.argtypes = [_i, _p, _p, _p, _p, _p, _p, _p, _i, _i64, _f, _f, _f, _f, _f, _f]
        L.orc_single1_backward.argtypes = [_i, _p, _p, _p, _p, _p, _p, _p, _i, _i64, _f, _f, _f, _f]
        L.orc_hfam_forward.argtypes = [_i, _p, _p, _p, _f, _p, _i, _i, _p, _p, _p, _p, _i, _i64,
                                       _f, _f, _f]
        L.orc_hfam_backward.argtypes = [_i, _p, _p, _f, _p, _i, _i, _p, _p, _p, _p, _i, _i64, _f,
                                        _f, _f, _f]
        L.orc_hfam_param_grads.argtypes = [_p, _p, _p, _p, _i, _i, _i, _i64, ctypes.c_double, _i,
                                           _p, _p]
        L.orc_gl_step_f32.argtypes = [_p, _p, _p, _i, _i64, _f, _i, _p]
        L.orc_gl_step_f64.argtypes = [_p, _p, _p, _i, _i64, ctypes.c_double, _i, _p]
        L.orc_glmulti_forward.argtypes = [_p, _p, _p, _p, _p, _p, _p, _p, _i, _i64, _f, _f]
        L.orc_glmulti_backward.argtypes = [_i, _p, _p, _p, _p, _p, _p, _p, _i, _i64, _f, _f, _f]
        L.orc_glmulti_param_grads.argtypes = [_p, _p, _p, _p, _p, _i, _i64]
        L.orc_aligned_forward.argtypes = [_p, _p, _p, _p, _p, _p, _p, _i, _i64, _f, _f]
        L.orc_aligned_backward.argtypes = [_p, _p, _p, _p, _p, _p, _p, _i, _i64, _f, _f, _f, _f]
        L.orc_aligned_param_grads.argtypes = [_p, _p, _p, _p, _p, _p, _i, _i64]
        L.orc_euler_forward.argtypes = [_p, _p, _p, _p, _p, _p, _i, _i64] + [_f] * 8
        L.orc_euler_backward.argtypes = [_p, _p, _p, _p, _p, _p, _p, _p, _i, _i64] + [_f] * 6
        L.orc_num_threads.restype = _i
        L.orc_set_num_threads.argtypes = [_i]
        L.orc_set_num_threads.restype = None
        _lib = L
    return _lib


def ref_available():
    return os.path.exists(REF_PATH)


def ref():
    """The reference's own kernels compiled for the host (None if not built)."""
    global _ref
    if _ref is None and ref_available():
        R = ctypes.CDLL(REF_PATH)
        for name in ("ref_gl_forward", "ref_trap_forward"):
            getattr(R, name).argtypes = [_p, _p, _p, _p, _p, _i, _i, _f, _f, _f, _f]
        R.ref_gl1_forward.argtypes = [_p, _p, _p, _p, _p, _i, _i, _f, _f, _f, _f, _f]
        R.ref_predictor_forward.argtypes = [_p, _p, _p, _p, _p, _i, _i, _f, _f, _f, _f, _f, _f]
        for name in ("ref_gl_backward", "ref_trap_backward"):
            getattr(R, name).argtypes = [_p, _p, _p, _p, _p, _p, _p, _i, _i, _f, _f, _f, _f]
        R.ref_gl1_backward.argtypes = [_p, _p, _p, _p, _p, _p, _p, _i, _i, _f, _f, _f, _f, _f]
        R.ref_predictor_backward.argtypes = [_p, _p, _p, _p, _p, _p, _p, _i, _i, _f, _f, _f, _f, _f, _f]
        R.ref_trap1_forward.argtypes = [_p, _p, _p, _p, _p, _i, _i, _f, _f, _f, _f, _f]
        R.ref_trap1_backward.argtypes = [_p, _p, _p, _p, _p, _p, _p, _i, _i, _f, _f, _f, _f, _f]
        R.ref_predictor1_forward.argtypes = [_p, _p, _p, _p, _p, _i, _i, _f, _f, _f, _f, _f, _f]
        R.ref_predictor1_backward.argtypes = [_p, _p, _p, _p, _p, _p, _p, _i, _i, _f, _f, _f, _f, _f, _f]
        R.ref_lifeuler_forward.argtypes = [_p, _p, _p, _p, _i, _i, _f, _f, _f]
        R.ref_lifeuler_backward.argtypes = [_p, _p, _p, _p, _p, _p, _i, _i, _f, _f, _f]
        R.ref_vogl1_forward.argtypes = [_p] * 8 + [_i] * 4 + [_f, _f]
        R.ref_vogl1_backward.argtypes = [_i] + [_p] * 7 + [_i] * 4 + [_f] * 3
        R.ref_fagl1_forward.argtypes = [_p] * 6 + [_i] * 4 + [_f] * 3
        R.ref_fagl1_backward.argtypes = [_i] + [_p] * 6 + [_i] * 4 + [_f] * 4
        R.ref_vopred_forward.argtypes = [_p] * 7 + [_i] * 4 + [_f] * 3
        R.ref_vopred_backward.argtypes = [_p] * 7 + [_i] * 4 + [_f] * 4
        R.ref_weighted_sum_f32.argtypes = [_p, _p, _p, _i, _i]
        R.ref_weighted_sum_f64.argtypes = [_p, _p, _p, _i, _i]
        R.ref_glmulti_forward.argtypes = [_p, _p, _p, _p, _p, _p, _p, _p, _i, _i, _f, _f]
        R.ref_glmulti_backward.argtypes = [_i, _p, _p, _p, _p, _p, _p, _p, _i, _i, _f, _f, _f]
        R.ref_aligned_forward.argtypes = [_p, _p, _p, _p, _p, _p, _p, _i, _i, _f, _f]
        R.ref_aligned_backward.argtypes = [_p, _p, _p, _p, _p, _p, _p, _i, _i, _f, _f, _f, _f]
        R.ref_euler_forward.argtypes = [_p, _p, _p, _p, _p, _p, _i, _i] + [_f] * 8
        R.ref_euler_backward.argtypes = [_p] * 10 + [_i, _i] + [_f] * 6
        _ref = R
    return _ref


def num_threads():
    return int(lib().orc_num_threads())


def set_num_threads(n):
    """OpenMP threads for the oracle and the host build of the reference kernels."""
    lib().orc_set_num_threads(int(n))


def _c(a, dtype=np.float32):
    return np.ascontiguousarray(a, dtype=dtype)


def _ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def _empty(T, N):
    return np.empty((T, N), dtype=np.float32)


# ---------------------------------------------------------------------------------------
# single-order schemes (gl / trap / predictor / gl1 / trap1 / predictor1)
# ---------------------------------------------------------------------------------------
def single_forward(scheme, x, v0, w, tau, beta, th, h_beta=1.0, gamma1=1.0, impl="oracle"):
    x, v0, w = _c(x), _c(v0), _c(w)
    T, N = x.shape
    s, v = _empty(T, N), _empty(T, N)
    if impl == "oracle":
        lib().orc_single_forward(SCHEMES[scheme], _ptr(x), _ptr(v0), _ptr(w), _ptr(s), _ptr(v),
                                 T, N, tau, beta, th, h_beta, gamma1)
    elif scheme == "euler":
        ref().ref_lifeuler_forward(_ptr(x), _ptr(v0), _ptr(s), _ptr(v), T, N, tau, th, 0.0)
    else:
        R = ref()
        args = [_ptr(x), _ptr(v0), _ptr(w), _ptr(s), _ptr(v), T, N, tau, beta, th, 0.0]
        if scheme == "gl":
            R.ref_gl_forward(*args)
        elif scheme == "trap":
            R.ref_trap_forward(*args)
        elif scheme == "gl1":
            R.ref_gl1_forward(*args, h_beta)
        elif scheme == "trap1":
            R.ref_trap1_forward(*args, h_beta)
        elif scheme == "predictor1":
            R.ref_predictor1_forward(*args, h_beta, gamma1)
        else:
            R.ref_predictor_forward(*args, h_beta, gamma1)
    return s, v


def single_backward(scheme, gS, gV, x, v0, w, tau, beta, th, sg, h_beta=1.0, gamma1=1.0,
                    impl="oracle", spike=None, vseq=None):
    """Reference backward (recomputes the forward, truncated history gradient)."""
    gS, gV, x, v0, w = _c(gS), _c(gV), _c(x), _c(v0), _c(w)
    T, N = x.shape
    gx = _empty(T, N)
    gv0 = np.empty(N, dtype=np.float32)
    if impl == "oracle" and scheme in RECOMPUTE_BACKWARD:
        lib().orc_single1_backward(SCHEMES[scheme], _ptr(gS), _ptr(gV), _ptr(x), _ptr(v0), _ptr(w),
                                   _ptr(gx), _ptr(gv0), T, N, tau, th, sg, h_beta)
    elif impl == "oracle":
        if spike is None or vseq is None:
            spike, vseq = single_forward(scheme, x, v0, w, tau, beta, th, h_beta, gamma1)
        spike, vseq = _c(spike), _c(vseq)
        lib().orc_single_backward(SCHEMES[scheme], _ptr(gS), _ptr(gV), _ptr(spike), _ptr(vseq),
                                  _ptr(w), _ptr(gx), _ptr(gv0), T, N, tau, beta, th, sg,
                                  h_beta, gamma1)
    elif scheme == "euler":
        ref().ref_lifeuler_backward(_ptr(gS), _ptr(gV), _ptr(x), _ptr(v0), _ptr(gx), _ptr(gv0),
                                    T, N, tau, th, sg)
    else:
        R = ref()
        args = [_ptr(gS), _ptr(gV), _ptr(x), _ptr(v0), _ptr(w), _ptr(gx), _ptr(gv0), T, N,
                tau, beta, th, sg]
        if scheme == "gl":
            R.ref_gl_backward(*args)
        elif scheme == "trap":
            R.ref_trap_backward(*args)
        elif scheme == "gl1":
            R.ref_gl1_backward(*args, h_beta)
        elif scheme == "trap1":
            R.ref_trap1_backward(*args, h_beta)
        elif scheme == "predictor1":
            R.ref_predictor1_backward(*args, h_beta, gamma1)
        else:
            R.ref_predictor_backward(*args, h_beta, gamma1)
    return gx, gv0


# ---------------------------------------------------------------------------------------
# library glmulti (LIFFDEGLMultiFunction)
# ---------------------------------------------------------------------------------------
def glmulti_forward(x, v0, scale, W, tau, th, impl="oracle"):
    x, v0, scale, W = _c(x), _c(v0), _c(scale), _c(W)
    T, N = x.shape
    s, vpre, vhist, drift = (_empty(T, N) for _ in range(4))
    fn = lib().orc_glmulti_forward if impl == "oracle" else ref().ref_glmulti_forward
    fn(_ptr(x), _ptr(v0), _ptr(scale), _ptr(W), _ptr(s), _ptr(vpre), _ptr(vhist), _ptr(drift),
       T, N, tau, th)
    return {"spike": s, "vpre": vpre, "vhist": vhist, "drift": drift}


def glmulti_backward(full, gS, scale, W, vpre, tau, th, sg, impl="oracle"):
    gS, scale, W, vpre = _c(gS), _c(scale), _c(W), _c(vpre)
    T, N = gS.shape
    gx, gpre = _empty(T, N), _empty(T, N)
    gv0 = np.empty(N, dtype=np.float32)
    fn = lib().orc_glmulti_backward if impl == "oracle" else ref().ref_glmulti_backward
    fn(int(bool(full)), _ptr(gS), _ptr(scale), _ptr(W), _ptr(vpre), _ptr(gx), _ptr(gv0),
       _ptr(gpre), T, N, tau, th, sg)
    return gx, gv0, gpre


def glmulti_param_grads(gpre, drift, vhist):
    """grad_scale = sum_n gpre*drift, grad_W = -gpre @ vhist^T, accumulated in double."""
    gpre, drift, vhist = _c(gpre), _c(drift), _c(vhist)
    T, N = gpre.shape
    gs = np.empty(T, dtype=np.float64)
    gW = np.empty((T, T), dtype=np.float64)
    lib().orc_glmulti_param_grads(_ptr(gpre), _ptr(drift), _ptr(vhist), _ptr(gs), _ptr(gW), T, N)
    return gs, gW


def glmulti_step(x, v0, scale, W, gS, tau, th, sg, full, impl="oracle"):
    """Forward + backward of LIFFDEGLMultiFunction; returns every output and gradient."""
    fw = glmulti_forward(x, v0, scale, W, tau, th, impl)
    gx, gv0, gpre = glmulti_backward(full, gS, scale, W, fw["vpre"], tau, th, sg, impl)
    gs, gW = glmulti_param_grads(gpre, fw["drift"], fw["vhist"])
    return dict(fw, gx=gx, gv0=gv0, gpre=gpre, gscale=gs, gW=gW)


# ---------------------------------------------------------------------------------------
# aligned glmulti (AlignedGLMulti of examples/*/aligned_glmulti.py)
# ---------------------------------------------------------------------------------------
def aligned_forward(x, v0, a, w, tau, th, impl="oracle"):
    x, v0, a, w = _c(x), _c(v0), _c(a), _c(w)
    T, N = x.shape
    s, p, hist = _empty(T, N), _empty(T, N), _empty(T, N)
    fn = lib().orc_aligned_forward if impl == "oracle" else ref().ref_aligned_forward
    fn(_ptr(x), _ptr(v0), _ptr(a), _ptr(w), _ptr(s), _ptr(p), _ptr(hist), T, N, tau, th)
    return {"spike": s, "pred": p, "hist": hist}


def aligned_backward(g, a, w, p, tau, th, sg, rho=1.0, impl="oracle"):
    g, a, w, p = _c(g), _c(a), _c(w), _c(p)
    T, N = g.shape
    gx, ga = _empty(T, N), _empty(T, N)
    gv = np.empty(N, dtype=np.float32)
    fn = lib().orc_aligned_backward if impl == "oracle" else ref().ref_aligned_backward
    fn(_ptr(g), _ptr(a), _ptr(w), _ptr(p), _ptr(gx), _ptr(gv), _ptr(ga), T, N, tau, th, sg, rho)
    return gx, gv, ga


def aligned_param_grads(ga, hist, w, a):
    ga, hist, w, a = _c(ga), _c(hist), _c(w), _c(a)
    T, N = ga.shape
    gs = np.empty(T, dtype=np.float64)
    gw = np.empty((T, T), dtype=np.float64)
    lib().orc_aligned_param_grads(_ptr(ga), _ptr(hist), _ptr(w), _ptr(a), _ptr(gs), _ptr(gw), T, N)
    return gs, gw


def aligned_step(x, v0, a, w, g, tau, th, sg, rho=1.0, impl="oracle"):
    fw = aligned_forward(x, v0, a, w, tau, th, impl)
    gx, gv, ga = aligned_backward(g, a, w, fw["pred"], tau, th, sg, rho, impl)
    gs, gw = aligned_param_grads(ga, fw["hist"], w, a)
    return dict(fw, gx=gx, gv0=gv, ga=ga, gscale=gs, gW=gw)


# ---------------------------------------------------------------------------------------
# direct LIF-like Euler (direct_euler_cupy.py)
# ---------------------------------------------------------------------------------------
def euler_forward(x, z0, in_scale, gain, bias, tau, th, step, reset_strength, sdt, impl="oracle"):
    x, z0 = _c(x), _c(z0)
    T, N = x.shape
    s, zpre, sin_ = _empty(T, N), _empty(T, N), _empty(T, N)
    zf = np.empty(N, dtype=np.float32)
    fn = lib().orc_euler_forward if impl == "oracle" else ref().ref_euler_forward
    fn(_ptr(x), _ptr(z0), _ptr(s), _ptr(zpre), _ptr(sin_), _ptr(zf), T, N, in_scale, gain, bias,
       tau, th, step, reset_strength, sdt)
    return {"spike": s, "zpre": zpre, "sin": sin_, "zfinal": zf}


def euler_backward(gS, gzf, x, zpre, sin_, in_scale, gain, tau, step, sg, sdt, impl="oracle"):
    gS, x, zpre, sin_ = _c(gS), _c(x), _c(zpre), _c(sin_)
    T, N = x.shape
    gx = _empty(T, N)
    gz0 = np.empty(N, dtype=np.float32)
    gzf_arr = None if gzf is None else _c(gzf)
    if impl == "oracle":
        g3 = np.empty(3, dtype=np.float64)
        lib().orc_euler_backward(_ptr(gS), None if gzf_arr is None else _ptr(gzf_arr), _ptr(x),
                                 _ptr(zpre), _ptr(sin_), _ptr(gx), _ptr(gz0), _ptr(g3), T, N,
                                 in_scale, gain, tau, step, sg, sdt)
    else:
        g3f = np.zeros(3, dtype=np.float32)
        if gzf_arr is None:
            gzf_arr = np.zeros(N, dtype=np.float32)
        base = g3f.ctypes.data
        ref().ref_euler_backward(_ptr(gS), _ptr(gzf_arr), _ptr(x), _ptr(zpre), _ptr(sin_),
                                 _ptr(gx), _ptr(gz0), ctypes.c_void_p(base),
                                 ctypes.c_void_p(base + 4), ctypes.c_void_p(base + 8),
                                 T, N, in_scale, gain, tau, step, sg, sdt)
        g3 = g3f.astype(np.float64)
    return gx, gz0, g3


# ---------------------------------------------------------------------------------------
# history family with per-sample tables: VO-GL1, FAGL1, VO-PREDICTOR
# (fde_cupy_kernels_all.py:1594-1843, :1200-1500, :1017-1198)
# ---------------------------------------------------------------------------------------
HFAM = {"vogl1": 0, "fagl1": 0, "vopred": 1}


def hfam_forward(kind, x, v0, scale, W, B, tau, th, hb=1.0, rm=0.0, impl="oracle"):
    """kind in vogl1 / fagl1 / vopred; scale None for fagl1 (uses hb); per-sample tables when
    W has three dimensions.  Returns spike, vpre, hsrc (v_hist or drift) and aux (drift for
    the GL kinds, drift + history for vopred; oracle only)."""
    x, v0, W = _c(x), _c(v0), _c(W)
    T, N = x.shape
    per_batch = int(W.ndim == 3)
    sc = None if scale is None else _c(scale)
    s, vpre, hsrc, aux = (_empty(T, N) for _ in range(4))
    if impl == "oracle":
        lib().orc_hfam_forward(HFAM[kind], _ptr(x), _ptr(v0), None if sc is None else _ptr(sc),
                               hb, _ptr(W), per_batch, B, _ptr(s), _ptr(vpre), _ptr(hsrc),
                               _ptr(aux), T, N, tau, th, rm)
        return {"spike": s, "vpre": vpre, "hsrc": hsrc, "aux": aux}
    R = ref()
    if kind == "vogl1":
        R.ref_vogl1_forward(_ptr(x), _ptr(v0), _ptr(sc), _ptr(W), _ptr(s), _ptr(vpre), _ptr(hsrc),
                            _ptr(aux), T, N, B, per_batch, tau, th)
    elif kind == "fagl1":
        R.ref_fagl1_forward(_ptr(x), _ptr(v0), _ptr(W), _ptr(s), _ptr(vpre), _ptr(hsrc), T, N, B,
                            per_batch, tau, hb, th)
    else:
        R.ref_vopred_forward(_ptr(x), _ptr(v0), _ptr(sc), _ptr(W), _ptr(s), _ptr(vpre), _ptr(hsrc),
                             T, N, B, per_batch, tau, th, rm)
    return {"spike": s, "vpre": vpre, "hsrc": hsrc}


def hfam_backward(kind, full, gS, vpre, scale, W, B, tau, th, sg, hb=1.0, rm=0.0, impl="oracle"):
    gS, vpre, W = _c(gS), _c(vpre), _c(W)
    T, N = gS.shape
    per_batch = int(W.ndim == 3)
    sc = None if scale is None else _c(scale)
    gx, gpre = _empty(T, N), _empty(T, N)
    gv0 = np.empty(N, dtype=np.float32)
    if impl == "oracle":
        mode = 2 if kind == "vopred" else (1 if full else 0)
        lib().orc_hfam_backward(mode, _ptr(gS), None if sc is None else _ptr(sc), hb, _ptr(W),
                                per_batch, B, _ptr(vpre), _ptr(gx), _ptr(gv0), _ptr(gpre), T, N,
                                tau, th, sg, rm)
    else:
        R = ref()
        if kind == "vogl1":
            R.ref_vogl1_backward(int(full), _ptr(gS), _ptr(sc), _ptr(W), _ptr(vpre), _ptr(gx),
                                 _ptr(gv0), _ptr(gpre), T, N, B, per_batch, tau, th, sg)
        elif kind == "fagl1":
            R.ref_fagl1_backward(int(full), _ptr(gS), _ptr(W), _ptr(vpre), _ptr(gx), _ptr(gv0),
                                 _ptr(gpre), T, N, B, per_batch, tau, hb, th, sg)
        else:
            R.ref_vopred_backward(_ptr(gS), _ptr(sc), _ptr(W), _ptr(vpre), _ptr(gx), _ptr(gv0),
                                  _ptr(gpre), T, N, B, per_batch, tau, th, sg, rm)
    return gx, gv0, gpre


def hfam_param_grads(G, V, E, scale, per_batch, B, sign, lower_only):
    """(gs, gW) as float64 arrays: gs[t,b] = sum G*E over sample b (None if E is None),
    gW[t,b,i] = sign * sum G*scale*V (per-sample layout [T,B,T] / [T,T])."""
    G, V = _c(G), _c(V)
    T, N = G.shape
    Ec = None if E is None else _c(E)
    sc = None if scale is None else _c(scale)
    gs = np.zeros((T, B) if per_batch else T, dtype=np.float64)
    gW = np.zeros((T, B, T) if per_batch else (T, T), dtype=np.float64)
    lib().orc_hfam_param_grads(_ptr(G), _ptr(V), None if Ec is None else _ptr(Ec),
                               None if sc is None else _ptr(sc), int(per_batch), B, T, N,
                               float(sign), int(lower_only), _ptr(gs), _ptr(gW))
    return (None if E is None else gs), gW


def hfam_params(kind, gpre, hsrc, drift, scale, W, B, lower_only_batch=True):
    """(grad_scale, grad_weights) in double as the reference Functions form them:
    VO-GL1 sum G*drift and -G@v_hist^T (:1829-1838); FAGL1 -G@v_hist^T, lower triangle only
    per sample (:1478-1497; the PyTorch Function keeps every entry: lower_only_batch=False);
    VO-PREDICTOR sum G*(drift + W@drift) and (G*scale)@drift^T (:1167-1181) -- hsrc is the
    drift for VO-PREDICTOR."""
    W = np.asarray(W)
    per_batch = W.ndim == 3
    if kind == "vogl1":
        return hfam_param_grads(gpre, hsrc, drift, None, per_batch, B, -1.0, 0)
    if kind == "fagl1":
        return None, hfam_param_grads(gpre, hsrc, None, None, per_batch, B, -1.0,
                                      int(per_batch and lower_only_batch))[1]
    _, gW = hfam_param_grads(gpre, hsrc, None, scale, per_batch, B, 1.0, 0)
    T, N = gpre.shape
    F = N // B
    G = np.asarray(gpre, np.float64).reshape(T, B, F)
    D = np.asarray(hsrc, np.float64).reshape(T, B, F)
    Wd = W.astype(np.float64)
    hist = np.einsum("tbi,ibf->tbf", Wd, D) if per_batch else np.einsum("ti,ibf->tbf", Wd, D)
    gsb = np.sum(G * (D + hist), axis=2)
    return (gsb if per_batch else gsb.sum(axis=1)), gW


# ---------------------------------------------------------------------------------------
# multi-term GL integrator of the SNN wrapper path (solver.py:2905-3002, :3270-3369)
# ---------------------------------------------------------------------------------------
def gl_step(f, hist, coef, c0_inv, chunk):
    """One integrator step: c0_inv * (f - conv) over hist [L, S] with coefficients coef[L]
    (see orc_gl_step_*; chunk > 0 weighted_sum chunks, 0 one chain, < 0 PyTorch loop)."""
    dt = np.asarray(f).dtype
    f = np.ascontiguousarray(f).reshape(-1)
    S = f.size
    hist = np.ascontiguousarray(hist, dtype=dt).reshape(-1, S)
    coef = np.ascontiguousarray(coef, dtype=dt)
    out = np.empty_like(f)
    fn = lib().orc_gl_step_f32 if dt == np.float32 else lib().orc_gl_step_f64
    fn(_ptr(f), _ptr(hist), _ptr(coef), hist.shape[0], S, float(c0_inv), int(chunk), _ptr(out))
    return out


def weighted_sum_ref(coeff, history):
    """The reference's weighted_sum kernel source compiled for the host."""
    dt = np.asarray(history).dtype
    history = np.ascontiguousarray(history)
    L, S = history.shape
    coeff = np.ascontiguousarray(coeff, dtype=dt)
    out = np.empty(S, dtype=dt)
    fn = ref().ref_weighted_sum_f32 if dt == np.float32 else ref().ref_weighted_sum_f64
    fn(_ptr(coeff), _ptr(history), _ptr(out), L, S)
    return out


def glmulti_integrate(f_of, y0, c_tilde, c0_inv, T, memory=None, chunk=96):
    """forward_glmulti_cupy (solver.py:3314-3362) for one integrated component given the
    coefficient table: f_of(k, y_current) -> f_k (numpy), y0 the initial state.  Returns the
    list of states y_1..y_T.  chunk as the reference's history_chunk_size (<= 0: PyTorch
    loop)."""
    kchunk = chunk if chunk > 0 else -1
    hist, y = [], y0
    for k in range(T):
        f = f_of(k, y)
        mem = k + 1 if memory in (None, -1) else min(memory, k + 1)
        start = max(0, k + 1 - mem)
        rows = hist[start:k] if k > start else []
        coef = np.array([c_tilde[k + 1 - j] for j in range(start, start + len(rows))], f.dtype)
        H = np.stack(rows) if rows else np.zeros((0, f.size), f.dtype)
        y = gl_step(f, H, coef, c0_inv, kchunk).reshape(f.shape)
        hist.append(y)
    return hist


def glmulti_adjoint(vjp_of, adj0, c_tilde, c0_inv, steps, memory=None):
    """backward_glmulti_cupy's update (solver.py:2958-2995) for one component: vjp_of(k,
    adj) -> vjp_y; rows 0..k of the adjoint history with c~[k+1-j], one fma chain."""
    hist = [adj0]
    adj = adj0
    for k in range(steps - 1):
        f = vjp_of(k, adj)
        mem = k + 1 if memory in (None, -1) else min(memory, k + 1)
        start = max(0, k + 1 - mem)
        rows = hist[start:k + 1]
        coef = np.array([c_tilde[k + 1 - j] for j in range(start, k + 1)], f.dtype)
        adj = gl_step(f, np.stack(rows), coef, c0_inv, 0).reshape(f.shape)
        hist.append(adj)
    return adj
