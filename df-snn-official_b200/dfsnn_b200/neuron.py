"""LIFNeuronFDE host mirror for the B200 multi-step path.

Same constructor signature, parameters/buffers (state_dict keys) and multi-step forward
contract as spikeDE_dis.neuron.LIFNeuronFDE (spikeDE_dis/neuron.py:1058-2270) for the
schemes of the hot path -- glmulti, gl, gl1 (truncated and full history), trap, predictor,
trap1, predictor1, euler, fagl1, vogl1, vopredictor -- dispatching to the
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

_NATIVE_METHODS = ("glmulti", "gl", "gl1", "trap", "predictor", "trap1", "predictor1", "euler",
                   "fagl1", "vogl1", "vopredictor")
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
        if self.history_grad_mode not in ("approx", "full"):
            raise ValueError("history_grad_mode must be 'approx' or 'full'")
        self._init_history_methods(vo_solver, vo_residual_mix, attn_dim, attn_temperature,
                                   attn_mode, attn_init, attn_stats_interval, name)
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

    def _init_history_methods(self, vo_solver, vo_residual_mix, attn_dim, attn_temperature,
                              attn_mode, attn_init, attn_stats_interval, name):
        """Variable-order and attention settings (neuron.py:1165-1221): the same validation,
        and for method='fagl1' the two bias-free [attn_dim, 2] projections of the attention
        descriptor, initialised from their own seed (1729 + the code points of `name`) so the
        rest of the model's RNG stream is untouched -- 'zero_q': Q = 0, K Xavier-uniform;
        'orthogonal_zero_score': four entries of magnitude sqrt(4/3) on distinct output rows
        (Q on two, K on two), so Q^T K = 0 and the first attention rows are uniform."""
        self.vo_solver = vo_solver
        self.vo_residual_mix = float(vo_residual_mix)
        self.attn_dim = int(attn_dim)
        self.attn_temperature = float(attn_temperature)
        self.attn_mode = str(attn_mode)
        self.attn_init = str(attn_init)
        self.attn_stats_interval = int(attn_stats_interval)
        if self.attn_dim <= 0:
            raise ValueError("attn_dim must be positive")
        if self.attn_temperature <= 0.0:
            raise ValueError("attn_temperature must be positive")
        if self.attn_mode not in ("batch_shared", "per_sample"):
            raise ValueError("attn_mode must be 'batch_shared' or 'per_sample'")
        if self.attn_init not in ("zero_q", "orthogonal_zero_score"):
            raise ValueError("attn_init must be 'zero_q' or 'orthogonal_zero_score'")
        if self.attn_stats_interval <= 0:
            raise ValueError("attn_stats_interval must be positive")
        if self.method == "fagl1" and self.attn_init == "orthogonal_zero_score" and self.attn_dim < 4:
            raise ValueError("orthogonal_zero_score requires attn_dim >= 4")
        if self.vo_solver not in ("abm", "l1", "abm_pc"):
            raise ValueError(f"Unsupported variable-order solver: {self.vo_solver}")
        if self.method == "fagl1" and self.beta_learnable:
            raise ValueError("method='fagl1' uses a fixed fractional order")
        self.fagl_q_proj = self.fagl_k_proj = None
        if self.method == "fagl1":
            seed = 1729 + sum(ord(c) for c in str(name))
            with torch.random.fork_rng(devices=[]):
                torch.manual_seed(seed)
                q = nn.Linear(2, self.attn_dim, bias=False)
                k = nn.Linear(2, self.attn_dim, bias=False)
                if self.attn_init == "zero_q":
                    nn.init.zeros_(q.weight)
                    nn.init.xavier_uniform_(k.weight)
                else:
                    nn.init.zeros_(q.weight)
                    nn.init.zeros_(k.weight)
                    rows = torch.randperm(self.attn_dim)
                    signs = torch.randint(0, 2, (4,)).mul_(2).sub_(1)
                    gain = math.sqrt(4.0 / 3.0)
                    for j, (proj, col) in enumerate(((q, 0), (q, 1), (k, 0), (k, 1))):
                        proj.weight.data[rows[j], col] = gain * signs[j]
            q._skip_direct_fde_init = True
            k._skip_direct_fde_init = True
            self.fagl_q_proj, self.fagl_k_proj = q, k
        self._fagl_stats_counter = 0
        self._fagl_static_cache = {}
        self._last_attention_entropy = None

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
        """Dispatch as neuron.py:1718-1763: gl1 with history_grad_mode='full' and fagl1 run the
        FAGL1 Functions (backend 'cupy': LIFFDEFAGL1Function, else LIFFDEFAGL1TorchFunction);
        vogl1 / vopredictor need a beta_schedule ([T], [T, B] or a dict with scale and
        weights) and run their Functions with vo_solver='abm'; the other solvers, like
        single-step mode, are the reference's per-step PyTorch path and are not provided."""
        if self.method not in _NATIVE_METHODS:
            raise NotImplementedError(f"method={self.method!r} is outside the B200 hot path")
        if not x_seq.is_cuda:
            raise RuntimeError("the B200 LIFNeuronFDE path requires CUDA input")
        if self.method == "gl1" and self.history_grad_mode == "full":
            if beta_schedule is not None:
                raise ValueError("method='gl1' rejects beta_schedule")
            return self._multi_step_forward_fagl1_function(
                x_seq, self._build_gl1_causal_weights(x_seq.shape[0], x_seq.device), True)
        if self.method == "fagl1":
            if beta_schedule is not None:
                raise ValueError("method='fagl1' uses a fixed order and rejects beta_schedule")
            return self._multi_step_forward_fagl1_function(
                x_seq, self._build_fagl1_weights(x_seq), self.history_grad_mode == "full")
        if self.method in ("vopredictor", "vogl1"):
            if beta_schedule is None:
                raise ValueError(f"method='{self.method}' requires beta_schedule")
            beta_values = beta_schedule["beta"] if isinstance(beta_schedule, dict) else beta_schedule
            if beta_values.shape[0] != x_seq.shape[0]:
                raise ValueError(f"beta_schedule has {beta_values.shape[0]} time values, "
                                 f"but input has {x_seq.shape[0]} time steps")
            if self.backend != "cupy" or self.vo_solver != "abm":
                raise NotImplementedError(
                    f"method={self.method!r} with backend={self.backend!r}, "
                    f"vo_solver={self.vo_solver!r} is the reference's per-step PyTorch path")
            return self._multi_step_forward_variable_order(x_seq, beta_schedule)
        if self.method == "glmulti":
            return self._multi_step_forward_glmulti(x_seq)
        return self._multi_step_forward_native(x_seq)

    # -- FAGL1 / GL1 full history / variable order (neuron.py:1790-2061) ----------------
    def _build_gl1_causal_weights(self, time_steps, device):
        """[T, T] GL1 history rows W[t, i] = c_{t-i} (i < t) for the neuron's fixed beta,
        coefficients accumulated in Python floats (double) and rounded once, as
        neuron.py:1880-1896."""
        beta = self._beta_value()
        c = [1.0]
        for lag in range(1, time_steps + 1):
            c.append((1.0 - (1.0 + beta) / float(lag)) * c[-1])
        lag = [[t - i if i < t else 0 for i in range(time_steps)] for t in range(time_steps)]
        table = torch.tensor([0.0] + c[1:], dtype=torch.float32)
        return table[torch.tensor(lag)].to(device)

    def _build_fagl1_weights(self, x_seq):
        """Per-sample (or batch-shared) causal attention rows times the fixed-order GL rows
        (neuron.py:1790-1866): descriptor (mean/rms, log rms) of each time step's input,
        scores = Q K^T / (sqrt(attn_dim) * temperature), a causal softmax, then
        W[t, ., i] = p[t, ., i] * t * c_{t-i}.  The mean normalised attention entropy is
        refreshed every attn_stats_interval calls."""
        if self.fagl_q_proj is None or self.fagl_k_proj is None:
            raise RuntimeError("FAGL1 attention projections are not initialized")
        xf = x_seq.float()
        dims = tuple(range(1, xf.dim())) if self.attn_mode == "batch_shared" else \
            tuple(range(2, xf.dim()))
        var, mean = torch.var_mean(xf, dim=dims, unbiased=False)
        rms = torch.sqrt((var + mean.square()).clamp_min(1e-8))
        desc = torch.stack((mean / (rms + 1e-6), torch.log(rms.clamp_min(1e-6))), dim=-1)
        q = self.fagl_q_proj(desc)
        k = self.fagl_k_proj(desc)
        if self.attn_mode == "batch_shared":
            scores = torch.mm(q, k.transpose(0, 1))
        else:
            scores = torch.bmm(q.permute(1, 0, 2), k.permute(1, 2, 0)).permute(1, 0, 2)
        scores = scores / (math.sqrt(float(self.attn_dim)) * self.attn_temperature)
        T = x_seq.shape[0]
        beta = self._beta_value()
        key = (x_seq.device.type, x_seq.device.index, T, beta)
        st = self._fagl_static_cache.get(key)
        if st is None:
            coef, c = [1.0], 1.0
            for lag in range(1, T + 1):
                c *= 1.0 - (1.0 + beta) / float(lag)
                coef.append(c)
            gl = torch.tensor(coef, device=x_seq.device, dtype=torch.float32)
            t_idx = torch.arange(T, device=x_seq.device)
            causal = t_idx.unsqueeze(0) < t_idx.unsqueeze(1)
            st = {"t_index": t_idx, "causal": causal,
                  "safe_causal": causal | ((t_idx == 0)[:, None] & (t_idx == 0)[None, :]),
                  "gl_kernel": gl[(t_idx[:, None] - t_idx[None, :]).clamp_min(0)] * causal,
                  "entropy_normalizer": torch.log(t_idx[2:].float())}
            self._fagl_static_cache[key] = st
        t_idx, causal, safe = st["t_index"], st["causal"], st["safe_causal"]
        if self.attn_mode == "batch_shared":
            prob = torch.softmax(scores.masked_fill(~safe, -torch.inf), dim=-1) * causal
            weights = prob * t_idx[:, None] * st["gl_kernel"]
        else:
            prob = torch.softmax(scores.masked_fill(~safe[:, None, :], -torch.inf), dim=-1)
            prob = prob * causal[:, None, :]
            weights = prob * t_idx[:, None, None] * st["gl_kernel"][:, None, :]
        if T > 2 and self._fagl_stats_counter % self.attn_stats_interval == 0:
            with torch.no_grad():
                p = prob.detach()
                ent = -(p.clamp_min(1e-8).log() * p).sum(dim=-1)
                norm = st["entropy_normalizer"]
                if self.attn_mode == "per_sample":
                    norm = norm[:, None]
                self._last_attention_entropy = (ent[2:] / norm).mean()
        elif T <= 2 and self._last_attention_entropy is None:
            self._last_attention_entropy = weights.new_tensor(1.0)
        self._fagl_stats_counter += 1
        return weights

    def get_attention_stats(self):
        if self.method != "fagl1" or self._last_attention_entropy is None:
            return None
        return {"entropy": float(self._last_attention_entropy.cpu())}

    def _multi_step_forward_fagl1_function(self, x_seq, weights, full):
        fn = _kernels.LIFFDEFAGL1Function if self.backend == "cupy" else \
            _kernels.LIFFDEFAGL1TorchFunction
        x_flat, v_init = self._initial_voltage_flat(x_seq)
        h_beta = float(self.h) ** self._beta_value()
        spike_flat = fn.apply(x_flat, v_init, weights, float(self.get_tau()), h_beta,
                              float(self.threshold), float(self.surrogate_grad_scale),
                              x_seq.shape[1], full)
        self.v = self._reset_state(x_seq[0])
        self.k = x_seq.shape[0]
        return spike_flat.reshape_as(x_seq)

    def _multi_step_forward_variable_order(self, x_seq, beta_schedule):
        if isinstance(beta_schedule, dict):
            scale, weights = beta_schedule["scale"], beta_schedule["weights"]
        else:
            build = _sched.build_vogl1_schedule if self.method == "vogl1" else \
                _sched.build_vopredictor_schedule
            terms = build(beta_schedule, self.h)
            scale, weights = terms["scale"], terms["weights"]
        x_flat = x_seq.flatten(1)
        if isinstance(self.v, torch.Tensor) and self.v.shape == x_seq[0].shape:
            v_init = self.v.flatten().to(dtype=torch.float32)
        else:
            v_init = self._reset_state(x_flat[0].float())
        tau, th, sg = float(self.get_tau()), float(self.threshold), float(self.surrogate_grad_scale)
        if self.method == "vogl1":
            spike_flat = _kernels.LIFFDEVOGL1Function.apply(
                x_flat, v_init, scale, weights, tau, th, sg, x_seq.shape[1],
                self.history_grad_mode == "full")
        else:
            spike_flat = _kernels.LIFFDEVOPREDICTORFunction.apply(
                x_flat, v_init, scale, weights, tau, th, sg, self.vo_residual_mix, x_seq.shape[1])
        self.v = self._reset_state(x_seq[0])
        self.k = x_seq.shape[0]
        return spike_flat.reshape_as(x_seq)

    @staticmethod
    def build_vogl1_schedule(beta_schedule, step_size):
        return _sched.build_vogl1_schedule(beta_schedule, step_size)

    @staticmethod
    def build_vopredictor_schedule(beta_schedule, step_size):
        return _sched.build_vopredictor_schedule(beta_schedule, step_size)

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
