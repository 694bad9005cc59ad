"""LIFNeuronFDE host mirror for the B200 multi-step path.

Same constructor signature, parameters/buffers (state_dict keys) and multi-step forward
contract as spikeDE_dis.neuron.LIFNeuronFDE (spikeDE_dis/neuron.py:1058-2270) for the
schemes of the hot path -- glmulti, gl, gl1, trap, predictor, trap1, predictor1 -- dispatching to the
autograd Functions of dfsnn_b200.fde_kernels exactly as the reference's
_multi_step_forward_glmulti_cupy (:1992-2007) and _multi_step_forward_cupy (:2091-2270)
dispatch to fde_cupy_kernels_all.  Functions are looked up on the module at call time, so
dfsnn_b200.aligned_glmulti.install() rebinding LIFFDEGLMultiFunction takes effect as it
does in the reference examples.

Single-step mode and backend='torch' are the reference's CPU/PyTorch implementation and
are not provided here (there is no CPU fallback on this path).
"""
import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import fde_kernels as _kernels
from . import schedule as _sched

_NATIVE_METHODS = ("glmulti", "gl", "gl1", "trap", "predictor", "trap1", "predictor1", "euler")
_ALL_METHODS = ("gl", "gl1", "fagl1", "vogl1", "predictor", "predictor1", "vopredictor", "trap",
                "trap1", "euler", "glmulti")


class LIFNeuronFDE(nn.Module):
    def __init__(self, tau=0.5, threshold=1.0, surrogate_alpha=4.0, surrogate_function="sigmoid",
                 tau_learnable=False, method="gl", beta=0.5, beta_learnable=False, batchsize=32,
                 T=16, step_size=1.0, memory=-1, name="", step_mode="s", v_reset=0.,
                 store_v_seq=False, backend="torch", detach_grad_steps=1, reset_mode=None,
                 detach_reset=False, decay_input=True, multi_beta=None, multi_coefficient=None,
                 learn_coefficient=True, coefficient_constraint="none",
                 shared_multi_coefficient=None, coefficient_update_interval=1,
                 glmulti_history_grad="truncated", history_grad_mode="approx", vo_solver="abm",
                 vo_reset_in_drift=False, vo_residual_mix=0.0, attn_dim=4, attn_temperature=1.0,
                 attn_mode="per_sample", attn_init="orthogonal_zero_score", attn_stats_interval=32,
                 surrogate_grad_scale=None, surrogate_opt=None):
        super().__init__()
        if surrogate_grad_scale is not None:
            surrogate_alpha = surrogate_grad_scale
        if surrogate_opt is not None:
            surrogate_function = {"sigmoid_surrogate": "sigmoid", "arctan_surrogate": "arctan",
                                  "piecewise_linear_surrogate": "piecewise_linear",
                                  "gaussian_surrogate": "gaussian"}.get(surrogate_opt, "sigmoid")
        if method not in _ALL_METHODS:
            raise ValueError(f"unsupported method: {method}")
        # BaseNeuron state (neuron.py:15-60)
        self.initial_tau = tau
        if tau_learnable:
            self.tau_param = nn.Parameter(torch.tensor(0.0), requires_grad=True)
        else:
            self.tau_param = None
            self.tau = tau
        self.threshold = threshold
        self.surrogate_grad_scale = surrogate_alpha
        self.surrogate_alpha = surrogate_alpha
        self.surrogate_function = surrogate_function
        self.tau_learnable = tau_learnable
        # LIFNeuronFDE state (neuron.py:1150-1318)
        self.method = method
        self.T = T
        self.name = name
        self.h = step_size
        self.initial_beta = beta
        self.beta_learnable = beta_learnable
        if beta_learnable:
            b = max(1e-6, min(1.0 - 1e-6, beta))
            self.beta_param = nn.Parameter(torch.tensor(math.log(b / (1.0 - b))), requires_grad=True)
        else:
            self.beta_param = None
            self.beta = beta
        self.batchsize = batchsize
        self.step_mode = step_mode
        self.v_reset = v_reset
        self.store_v_seq = store_v_seq
        self.backend = backend
        self.detach_grad_steps = detach_grad_steps
        self.detach_reset = detach_reset
        self.decay_input = decay_input
        self.learn_coefficient = bool(learn_coefficient)
        self.coefficient_constraint = str(coefficient_constraint)
        self.coefficient_update_interval = int(coefficient_update_interval)
        self.glmulti_history_grad = str(glmulti_history_grad)
        self.history_grad_mode = str(history_grad_mode)
        self._coefficient_forward_count = 0
        if self.coefficient_constraint not in ("none", "softplus", "softmax"):
            raise ValueError("coefficient_constraint must be 'none', 'softplus', or 'softmax'")
        if self.coefficient_update_interval <= 0:
            raise ValueError("coefficient_update_interval must be positive")
        if self.glmulti_history_grad not in ("truncated", "full"):
            raise ValueError("glmulti_history_grad must be 'truncated' or 'full'")
        if self.method == "glmulti":
            if multi_beta is None or multi_coefficient is None:
                raise ValueError("method='glmulti' requires multi_beta and multi_coefficient.")
            if len(multi_beta) != len(multi_coefficient):
                raise ValueError("multi_beta and multi_coefficient must have the same length")
            mb = torch.tensor(multi_beta, dtype=torch.float32)
            if torch.any((mb <= 0.0) | (mb > 1.0)):
                raise ValueError("All multi_beta values must be in (0, 1].")
            self.register_buffer("multi_beta", mb)
            coef = torch.tensor(multi_coefficient, dtype=torch.float32)
            if self.learn_coefficient:
                if self.coefficient_constraint in ("softplus", "softmax") and torch.any(coef <= 0.0):
                    raise ValueError(f"{self.coefficient_constraint}-constrained coefficients "
                                     "must be initialized above zero.")
                if self.coefficient_constraint in ("softplus", "softmax"):
                    raw = (torch.log(torch.expm1(coef.clamp_min(1e-6)))
                           if self.coefficient_constraint == "softplus" else torch.log(coef))
                    if shared_multi_coefficient is not None:
                        if shared_multi_coefficient.shape != raw.shape:
                            raise ValueError("Shared coefficient parameter has the wrong shape.")
                        self.multi_coefficient_raw = shared_multi_coefficient
                    else:
                        self.multi_coefficient_raw = nn.Parameter(raw)
                    self.multi_coefficient = None
                else:
                    self.multi_coefficient = (shared_multi_coefficient
                                              if shared_multi_coefficient is not None
                                              else nn.Parameter(coef))
                    self.multi_coefficient_raw = None
            else:
                self.register_buffer("multi_coefficient", coef)
                self.multi_coefficient_raw = None
            self.register_buffer("_glmulti_basis", _sched.glmulti_basis(multi_beta, self.T))
        else:
            self.multi_beta = None
            self.multi_coefficient = None
            self.multi_coefficient_raw = None
            self._glmulti_basis = None
        self.reset_mode = reset_mode if reset_mode is not None else ("soft" if v_reset is None else "hard")
        self.memory = None if memory == -1 else memory
        self.weights = None
        self.h_beta = None
        self.k = 0
        self._initialized = False
        self.v = v_reset
        self.v_seq = None

    # -- parameters -----------------------------------------------------------------
    def get_tau(self):
        if self.tau_learnable:
            return self.initial_tau * (1 + torch.exp(self.tau_param))
        return self.tau

    def get_beta(self):
        if self.beta_learnable:
            return torch.sigmoid(self.beta_param).clamp(min=1e-6, max=1.0 - 1e-6)
        return self.beta

    def get_multi_coefficient(self):
        if self.method != "glmulti":
            return None
        if self.coefficient_constraint == "softplus" and self.learn_coefficient:
            return F.softplus(self.multi_coefficient_raw)
        if self.coefficient_constraint == "softmax" and self.learn_coefficient:
            return torch.softmax(self.multi_coefficient_raw, dim=0)
        return self.multi_coefficient

    def _beta_value(self):
        b = self.get_beta()
        return b.detach().item() if isinstance(b, torch.Tensor) else b

    def _reset_state(self, like):
        """A tensor shaped like `like` holding v_reset (float32 unless `like` says otherwise).

        The reference allocates and fills a fresh tensor on every reset and after every glmulti
        forward (one [N] fill each).  Here one filled tensor per shape is kept and handed out
        again while nobody has written to it (its version counter is unchanged); a tensor that
        was modified in place is replaced by a new one, never refilled, so tensors saved for a
        backward are never touched."""
        key = (tuple(like.shape), like.device, like.dtype)
        cache = self.__dict__.setdefault("_reset_cache", {})
        got = cache.get(key)
        if got is not None and got[0]._version == got[1]:
            return got[0]
        t = torch.full_like(like, float(self.v_reset)).detach()
        cache[key] = (t, t._version)
        return t

    def reset(self):
        self.k = 0
        if isinstance(self.v, torch.Tensor):
            self.v = self._reset_state(self.v)
        else:
            self.v = self.v_reset
        if self.store_v_seq:
            self.v_seq = None

    # -- schedules ---------------------------------------------------------------------
    def _build_glmulti_schedule(self, T, device):
        # Softplus-constrained (or unconstrained) masses: one native launch per direction
        # (GLMultiScheduleFunction, bit-identical forward); softmax keeps PyTorch's chain.
        fused = device.type == "cuda" and (self.coefficient_constraint != "softmax"
                                           or not self.learn_coefficient)
        if fused:
            if self.learn_coefficient and self.coefficient_constraint == "softplus":
                src, constraint = self.multi_coefficient_raw, 1
            else:
                src, constraint = self.multi_coefficient, 0
        else:
            src = self.get_multi_coefficient()
        if torch.is_grad_enabled() and self.learn_coefficient:
            update = self._coefficient_forward_count % self.coefficient_update_interval == 0
            self._coefficient_forward_count += 1
            if not update:
                src = src.detach()
        if T != self.T:
            raise ValueError(f"glmulti was initialized for T={self.T}, got T={T}")
        basis = self._glmulti_basis.to(device=device, dtype=torch.float32)
        key = (device.type, device.index)
        cache = self.__dict__.setdefault("_h_pow_cache", {})
        if key not in cache:
            cache[key] = _sched.h_pow_neg_beta(self.h, self.multi_beta, device)
        if fused:
            scale, weights = _sched.GLMultiScheduleFunction.apply(
                src.to(device), basis, cache[key], constraint)
            return {"scale": scale, "weights": weights}
        return _sched.build_glmulti_schedule(src, self.multi_beta, basis, self.h, T,
                                             h_pow=cache[key])

    def _compute_weights(self, T, device, dtype):
        beta = self._beta_value()
        if self.method in ("gl", "gl1"):
            return _sched.gl_weights(beta, T, device, dtype)
        if self.method in ("trap", "trap1"):                   # neuron.py:1431-1436
            return _sched.trap_weights(beta, T, device, dtype)
        if self.method in ("predictor", "predictor1"):
            return _sched.predictor_weights(beta, T, device, dtype)
        return None

    def initialize(self, v_mem):
        self.batchsize = v_mem.shape[0]
        self.weights = self._compute_weights(self.T, v_mem.device, v_mem.dtype)
        self._initialized = True
        return v_mem

    # -- forward -----------------------------------------------------------------------
    def forward(self, x, beta_schedule=None):
        if self.step_mode == "s":
            raise NotImplementedError("single-step mode is the reference's PyTorch path; the B200 "
                                      "path is multi-step (step_mode='m')")
        if self.step_mode != "m":
            raise ValueError(f"unsupported step_mode: {self.step_mode}")
        return self.multi_step_forward(x, beta_schedule=beta_schedule)

    def multi_step_forward(self, x_seq, beta_schedule=None):
        if self.method not in _NATIVE_METHODS:
            raise NotImplementedError(f"method={self.method!r} is outside the B200 hot path")
        if not x_seq.is_cuda:
            raise RuntimeError("the B200 LIFNeuronFDE path requires CUDA input")
        if self.method == "glmulti":
            return self._multi_step_forward_glmulti(x_seq)
        return self._multi_step_forward_native(x_seq)

    def _initial_voltage_flat(self, x_seq):
        x_flat = x_seq.flatten(1)
        if isinstance(self.v, torch.Tensor) and self.v.shape == x_seq[0].shape:
            return x_flat, self.v.flatten().float()
        return x_flat, self._reset_state(x_flat[0].float())

    def _multi_step_forward_glmulti(self, x_seq):
        T = x_seq.shape[0]
        terms = self._build_glmulti_schedule(T, x_seq.device)
        x_flat, v_init = self._initial_voltage_flat(x_seq)
        spike_flat = _kernels.LIFFDEGLMultiFunction.apply(
            x_flat, v_init, terms["scale"], terms["weights"], float(self.get_tau()),
            float(self.threshold), float(self.surrogate_grad_scale), x_seq.shape[1],
            self.glmulti_history_grad == "full")
        self.v = self._reset_state(x_seq[0])
        self.k = T
        return spike_flat.reshape_as(x_seq)

    def _v_float_to_tensor(self, x):
        if isinstance(self.v, float) or not isinstance(self.v, torch.Tensor):
            self.v = torch.full_like(x.data, float(self.v))
        elif self.v.shape[0] != x.shape[0]:
            if x.shape[0] < self.v.shape[0]:
                self.v = self.v[:x.shape[0]].contiguous()
            else:
                extra = torch.full((x.shape[0] - self.v.shape[0],) + self.v.shape[1:], self.v_reset,
                                   device=self.v.device, dtype=self.v.dtype)
                self.v = torch.cat([self.v, extra], dim=0)

    def _multi_step_forward_native(self, x_seq):
        original_shape = x_seq.shape
        T = x_seq.shape[0]
        x_flat = x_seq.flatten(1)
        if not self._initialized:
            self.initialize(x_seq[0])
        self._v_float_to_tensor(x_seq[0])
        v_flat = self.v.flatten(0)
        self.k = 0
        tau = self.get_tau()
        tau = tau.item() if isinstance(tau, torch.Tensor) else tau
        beta = self._beta_value()
        v_reset = self.v_reset if self.v_reset is not None else 0.0
        K = _kernels
        if self.method == "gl":
            s, v = K.LIFFDEGLFunction.apply(x_flat, v_flat, self.weights, tau, beta, self.threshold,
                                            v_reset, self.surrogate_grad_scale)
        elif self.method == "gl1":
            s, v = K.LIFFDEGL1Function.apply(x_flat, v_flat, self.weights, tau, beta, self.h,
                                             self.threshold, v_reset, self.surrogate_grad_scale)
        elif self.method == "trap":
            s, v = K.LIFFDETRAPFunction.apply(x_flat, v_flat, self.weights, tau, beta,
                                              self.threshold, v_reset, self.surrogate_grad_scale)
        elif self.method == "euler":                             # neuron.py:2247-2255
            s, v = K.LIFEulerFunction.apply(x_flat, v_flat, tau, self.threshold, v_reset,
                                            self.surrogate_grad_scale)
        elif self.method == "trap1":
            s, v = K.LIFFDETRAP1Function.apply(x_flat, v_flat, self.weights, tau, beta,
                                               self.threshold, v_reset, self.surrogate_grad_scale)
        elif self.method == "predictor1":
            h_beta, gamma1 = _sched.predictor_constants(beta, self.h)
            s, v = K.LIFFDEPREDICTOR1Function.apply(x_flat, v_flat, self.weights, tau, beta,
                                                    self.threshold, v_reset,
                                                    self.surrogate_grad_scale, h_beta, gamma1)
        else:
            h_beta, gamma1 = _sched.predictor_constants(beta, self.h)
            s, v = K.LIFFDEPREDICTORFunction.apply(x_flat, v_flat, self.weights, tau, beta,
                                                   self.threshold, v_reset,
                                                   self.surrogate_grad_scale, h_beta, gamma1)
        spike_seq = s.reshape(original_shape)
        v_seq = v.reshape(original_shape)
        if self.store_v_seq:
            self.v_seq = v_seq
        self.v = v_seq[-1].clone()
        self.k = T
        return spike_seq
