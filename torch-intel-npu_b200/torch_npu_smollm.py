"""Frozen SmolLM decoder layers with low-bit projections on B200 (drop-in for torch_npu_smollm).

Keeps the reference module's public surface (torch_npu_smollm.py): ``FrozenSmolLayer``
(modes fp16 / w8a16 / w4a16 / nf4a16, ``packed_weights``, ``fp16_projections``,
``corrections``; ``forward`` / ``prefill`` / ``decode``), ``SmolKVCache`` snapshots and
``FrozenSmolStack`` (``from_checkpoint``, ``forward`` / ``prefill`` / ``decode``).

What changes underneath the API:
* every projection is one ``lb_linear`` call (decode GEMV / tcgen05 GEMM with the
  rank-r correction fused), instead of a compiled NPU graph;
* RMSNorm (fused with the residual add that precedes it), RoPE, the KV append and
  one-token GQA attention are the library's own kernels and follow the reference's fp16
  staging (torch_npu_smollm.py:166-193); prefill attention uses PyTorch SDPA;
* dimensions and RoPE theta come from the config (the reference hard-wires the 135M
  shape, theta 1e5 and 64 positions; torch_npu_smollm.py:79-83, :111-116);
* corrections are accepted for every quantized mode (the reference accepts them for
  w8a16 only, torch_npu_smollm.py:90-93; the correction math is format independent);
* ``SmolKVCache`` snapshots share one preallocated device buffer; decoding from a stale
  snapshot copies the buffer first, so snapshots stay immutable as in the reference.
``SmolForCausalLM`` (not in the reference) adds the tied embedding / LM head and a
greedy ``generate`` whose decode step is one replayed CUDA graph (for a tensor-parallel
stack, graphs split at the NCCL all-reduces, which run eagerly between them).
"""
from dataclasses import dataclass, field
import json
from pathlib import Path

import torch
import torch.nn.functional as F

import lowbit_runtime as rt
from torch_npu_lowbit import DevicePackedWeight, PackedWeight, quantize_weight_device
from torch_npu_lowbit_correction import LowRankCorrection
from torch_npu_smollm_io import FrozenSmolIO

_STACKS = {'qkv': ('self_attn.q_proj.weight', 'self_attn.k_proj.weight', 'self_attn.v_proj.weight'),
           'gate_up': ('mlp.gate_proj.weight', 'mlp.up_proj.weight')}
_FUSE_Z_ROWS = 16
_ZP = 64   # columns of a row-parallel projection's z in the all-reduce buffer
_PROJECTIONS = ('self_attn.q_proj.weight', 'self_attn.k_proj.weight', 'self_attn.v_proj.weight',
                'self_attn.o_proj.weight', 'mlp.gate_proj.weight', 'mlp.up_proj.weight', 'mlp.down_proj.weight')
_NORMS = ('input_layernorm.weight', 'post_attention_layernorm.weight')
_WEIGHT_FORMATS = {'fp16': None, 'w8a16': 'int8', 'w4a16': 'int4', 'nf4a16': 'nf4'}


class _PiecewiseGraph:
    """A decode step of a tensor-parallel stack as CUDA graphs split at its all-reduces.

    While recording, the step runs once on a side stream under capture; each all-reduce
    (``all_reduce``) ends the graph being captured, is kept as an eager step on its buffer,
    and a new graph begins.  The graphs share one memory pool and ``replay`` runs them in
    capture order, so a buffer allocated in one graph and summed before the next keeps its
    address.  The NCCL calls themselves are never captured."""

    active = None   # the recorder in use while a step is being captured

    def __init__(self):
        self.pool = torch.cuda.graph_pool_handle()
        self.steps = []
        self.graph = None

    def _begin(self):
        self.graph = torch.cuda.CUDAGraph(keep_graph=True)   # kept for launch counting
        # thread-local: the process group's watchdog thread keeps querying its events
        self.graph.capture_begin(pool=self.pool, capture_error_mode='thread_local')

    def _end(self):
        self.graph.capture_end()
        self.steps.append(('graph', self.graph))
        self.graph = None

    def record(self, fn):
        """Capture ``fn()`` (the decode step) on the current stream; returns its result."""
        _PiecewiseGraph.active = self
        try:
            self._begin()
            out = fn()
            self._end()
        finally:
            _PiecewiseGraph.active = None
            if self.graph is not None:   # an error inside a capture: close it before raising
                try:
                    self.graph.capture_end()
                except RuntimeError:
                    pass
                self.graph = None
        return out

    def all_reduce(self, buf, group):
        self._end()
        self.steps.append(('all_reduce', buf, group))
        self._begin()

    def replay(self):
        import torch.distributed as dist
        for step in self.steps:
            if step[0] == 'graph':
                step[1].replay()
            else:
                dist.all_reduce(step[1], group=step[2])

    def graphs(self):
        return [s[1] for s in self.steps if s[0] == 'graph']


def _all_reduce(buf, group):
    """Sum ``buf`` over the tensor-parallel group, or record it as a split point of the
    piecewise decode graph being captured."""
    if _PiecewiseGraph.active is not None:
        _PiecewiseGraph.active.all_reduce(buf, group)
        return
    import torch.distributed as dist
    dist.all_reduce(buf, group=group)


def _projection_policy(mode, names):
    """torch_npu_smollm.py:31-37."""
    if (type(names) is not tuple or any(type(name) is not str for name in names)
            or len(set(names)) != len(names) or not set(names) <= set(_PROJECTIONS)):
        raise ValueError('fp16_projections requires a tuple of distinct SmolLM projection weight names')
    if names and (mode != 'w8a16' or len(names) == len(_PROJECTIONS)):
        raise ValueError('FP16 protection requires w8a16 with at least one INT8 projection; use mode=fp16 for all FP16')
    return frozenset(names)


@dataclass(frozen=True)
class SmolConfig:
    hidden: int
    intermediate: int
    heads: int
    kv_heads: int
    head_dim: int
    eps: float
    theta: float
    vocab: int
    layers: int

    @classmethod
    def from_dict(cls, config):
        """Llama-style SmolLM config (the reference requires exactly the 135M values)."""
        required = dict(model_type='llama', hidden_act='silu', attention_bias=False, mlp_bias=False)
        if any(config.get(k, v) != v for k, v in required.items()) or config.get('rope_scaling') is not None:
            raise ValueError('Requires a llama-style SmolLM configuration')
        hidden, heads = config['hidden_size'], config['num_attention_heads']
        kv = config.get('num_key_value_heads', heads)
        head_dim = config.get('head_dim', hidden // heads)   # explicit for tensor-parallel shards
        if heads % kv or head_dim != 64:
            raise ValueError('Requires head_dim 64 and grouped KV heads')
        return cls(hidden, config['intermediate_size'], heads, kv, head_dim, float(config.get('rms_norm_eps', 1e-5)),
                   float(config.get('rope_theta', 10000.0)), int(config.get('vocab_size', 49152)),
                   int(config.get('num_hidden_layers', 1)))

    def shapes(self):
        d, f, hd = self.hidden, self.intermediate, self.head_dim
        q, kv = self.heads * hd, self.kv_heads * hd
        return {'self_attn.q_proj.weight': (q, d), 'self_attn.k_proj.weight': (kv, d), 'self_attn.v_proj.weight': (kv, d),
                'self_attn.o_proj.weight': (d, q), 'mlp.gate_proj.weight': (f, d), 'mlp.up_proj.weight': (f, d),
                'mlp.down_proj.weight': (d, f), 'input_layernorm.weight': (d,), 'post_attention_layernorm.weight': (d,)}


def rope_tables(cfg, positions, device):
    """fp16 cos/sin [positions, head_dim] built like torch_npu_smollm.py:113-116."""
    hd = cfg.head_dim
    frequency = 1. / (cfg.theta ** (torch.arange(0, hd, 2).float() / hd))
    angles = torch.outer(torch.arange(positions).float(), frequency)
    angles = torch.cat((angles, angles), dim=-1)
    return angles.cos().half().to(device), angles.sin().half().to(device)


@dataclass(eq=False)
class _CacheStore:
    keys: torch.Tensor        # [B, kv_heads, max_pos, hd]
    values: torch.Tensor
    written: int              # longest prefix any snapshot has written


@dataclass(frozen=True, eq=False)
class SmolKVCache:
    """KV snapshot (torch_npu_smollm.py:547-555): positions [0, length) are valid."""
    _owner: object
    _sequence: object
    _store: _CacheStore = field(repr=False)
    length: int

    @property
    def keys(self):
        return self._store.keys[:, :, :self.length]

    @property
    def values(self):
        return self._store.values[:, :, :self.length]


class FrozenSmolLayer(torch.nn.Module):
    """One decoder layer on the GPU; constructor arguments follow torch_npu_smollm.py:74-117."""

    def __init__(self, config, weights, *, mode='w8a16', packed_weights=None, fp16_projections=(), corrections=None,
                 group_size=None, device=None, max_positions=None, tp_group=None, row_corrections=None):
        """``tp_group`` (a torch.distributed NCCL group) makes this the per-rank piece of a
        tensor-parallel layer: ``config``/``weights`` are the rank's shard (see
        smollm_parallel.shard_layer_weights) and ``row_corrections`` holds the row-parallel
        projections' (V shard, U) factors."""
        super().__init__()
        if mode not in _WEIGHT_FORMATS:
            raise ValueError('Requires fp16, w8a16, w4a16 or nf4a16')
        cfg = config if isinstance(config, SmolConfig) else SmolConfig.from_dict(config)
        self.config = cfg
        self._mode = mode
        weight_format = _WEIGHT_FORMATS[mode]
        self._fp16_projections = _projection_policy(mode, fp16_projections)
        shapes = cfg.shapes()
        if set(weights) != set(shapes):
            raise ValueError('Unexpected layer weight names')
        if corrections is not None and (type(corrections) is not dict or mode == 'fp16'
                                        or not set(corrections) <= set(_PROJECTIONS)
                                        or set(corrections) & self._fp16_projections
                                        or any(not isinstance(c, LowRankCorrection) or c.shape != shapes[n] or c.rank > 32
                                               for n, c in corrections.items())):
            raise ValueError('Corrections require matching rank<=32 factors on quantized, unprotected projections')
        if packed_weights is not None:
            if weight_format is None or type(packed_weights) is not dict or set(packed_weights) != set(_PROJECTIONS):
                raise ValueError('Prepared weights require all seven projections in a matching lowbit mode')
            for name, q in packed_weights.items():
                if (not isinstance(q, (PackedWeight, DevicePackedWeight)) or q.shape != shapes[name] or q.format != weight_format
                        or (weight_format == 'int8' and q.group_size != shapes[name][1])):
                    raise ValueError('Prepared weights require matching formats/shapes; W8 uses per-row scales')
        rt.require_cuda()
        self.device = rt.cuda_device(device)
        self.max_positions = max_positions or 4096
        self._proj = {}
        for name in _PROJECTIONS:
            w = weights[name]
            if not isinstance(w, torch.Tensor) or w.dtype not in (torch.float16, torch.bfloat16, torch.float32):
                raise ValueError('Preparation requires FP16/BF16/FP32 weights')
            n, k = shapes[name]
            if weight_format is None or name in self._fp16_projections:
                codes = w.detach().to(self.device, torch.float16).contiguous().view(torch.uint8).reshape(-1)
                entry = dict(fmt='fp16', group=k, codes=codes, scales=None, packed=None)
            elif packed_weights is not None:
                q = packed_weights[name]
                codes, scales = q.to_device(self.device)
                entry = dict(fmt=weight_format, group=q.group_size, codes=codes, scales=scales, packed=q)
            else:
                gs = group_size.get(name) if isinstance(group_size, dict) else group_size
                g = k if weight_format == 'int8' else (gs or 32)
                half = w.detach().to(self.device, torch.float16)   # reference quantizes w.float().half()
                codes, scales = quantize_weight_device(half, format=weight_format, group_size=g)
                entry = dict(fmt=weight_format, group=g, codes=codes, scales=scales, packed=None)
            entry.update(n=n, k=k, down=None, up=None)
            if corrections and name in corrections:
                down, up = corrections[name].tensors()
                entry['down'], entry['up'] = down.to(self.device), up.to(self.device)
            self._proj[name] = entry
        self._norm = {name: weights[name].detach().to(self.device, torch.float16).contiguous() for name in _NORMS}
        self._stacks = {key: self._stack(names) for key, names in _STACKS.items()}
        self._tp = tp_group
        self._row_corr = {}
        for name, (down, up) in (row_corrections or {}).items():
            # rank padded to _ZP with zero factors: z keeps a _ZP-column row in the exchange
            # buffer, and the z U^T product stays on the tensor-core path at prefill sizes
            # (its K must be a multiple of 64)
            r = down.shape[0]
            downp = torch.zeros(_ZP, down.shape[1], dtype=torch.float16, device=self.device)
            upp = torch.zeros(up.shape[0], _ZP, dtype=torch.float16, device=self.device)
            downp[:r] = down.to(self.device, torch.float16)
            upp[:, :r] = up.to(self.device, torch.float16)
            self._row_corr[name] = (downp, upp)
        self._owner = object()
        self.eval()

    mode = property(lambda self: self._mode)
    fp16_projections = property(lambda self: self._fp16_projections)

    @classmethod
    def from_checkpoint(cls, directory, *, layer_index=0, mode='w8a16', packed_weights=None, fp16_projections=(),
                        corrections=None, **options):
        """One layer of a SmolLM safetensors checkpoint directory (torch_npu_smollm.py:119-127);
        ``options`` are this class's GPU keywords (group_size, device, max_positions)."""
        from safetensors import safe_open
        _projection_policy(mode, fp16_projections)
        directory = Path(directory)
        config = json.loads((directory / 'config.json').read_text())
        if type(layer_index) is not int or not 0 <= layer_index < config.get('num_hidden_layers', 0):
            raise ValueError('Invalid layer index')
        prefix = f'model.layers.{layer_index}.'
        with safe_open(directory / 'model.safetensors', framework='pt', device='cpu') as file:
            weights = {name[len(prefix):]: file.get_tensor(name) for name in file.keys() if name.startswith(prefix)}
        return cls(config, weights, mode=mode, packed_weights=packed_weights, fp16_projections=fp16_projections,
                   corrections=corrections, **options)

    def reference_cpu(self, x, *, quantized=True, segment=None, normalized=None):
        """Not provided: the reference's staged CPU layer (torch_npu_smollm.py:142-193) is its
        test oracle, and this package has no CPU path -- its restatement lives with the
        tests, as test infrastructure (oracle/decoder_ref.py in the source tree)."""
        raise NotImplementedError('reference_cpu is the CPU test oracle; this package runs on the GPU only')

    def _stack(self, names):
        """q/k/v (or gate/up) as one decode-GEMV launch (lb_linear_stacked): rows stacked in
        one code buffer (the single-projection entries become views of it), corrections as
        one block-diagonal correction of rank 32 per projection.  None when the projections
        differ in format or group (e.g. an fp16 exception)."""
        ents = [self._proj[n] for n in names]
        if len({(e['fmt'], e['group'], e['k']) for e in ents}) != 1:
            return None
        k = ents[0]['k']
        codes = torch.cat([e['codes'] for e in ents])
        scales = None if ents[0]['scales'] is None else torch.cat([e['scales'] for e in ents])
        off_c = off_s = 0
        for e in ents:   # share the stacked storage (offsets are 16-byte multiples here)
            nc, ns = e['codes'].numel(), 0 if scales is None else e['scales'].numel()
            if off_c % 16 == 0 and (off_s * 2) % 16 == 0:
                e['codes'] = codes[off_c:off_c + nc]
                if scales is not None:
                    e['scales'] = scales[off_s:off_s + ns]
            off_c, off_s = off_c + nc, off_s + ns
        n = sum(e['n'] for e in ents)
        down = up = None
        if any(e['down'] is not None for e in ents):
            rank = 32 * len(ents)
            down = torch.zeros(rank, k, dtype=torch.float16, device=self.device)
            up = torch.zeros(n, rank, dtype=torch.float16, device=self.device)
            row = 0
            for i, e in enumerate(ents):
                if e['down'] is not None:
                    r = e['down'].shape[0]
                    down[32 * i:32 * i + r] = e['down']
                    up[row:row + e['n'], 32 * i:32 * i + r] = e['up']
                row += e['n']
        return dict(fmt=ents[0]['fmt'], group=ents[0]['group'], n=n, k=k, codes=codes, scales=scales, down=down,
                    up=up, widths=[e['n'] for e in ents])

    def _stacked(self, key, x, residual=None):
        """The stacked launch when it applies (decode batch <= 64), else None."""
        st = self._stacks.get(key)
        if st is None or rt.linear_select(st['fmt'], st['group'], x.shape[0], st['n'], st['k']) != 'gemv':
            return None
        return rt.linear_stacked(x, st['fmt'], st['group'], st['n'], st['codes'], st['scales'], down=st['down'],
                                 up=st['up'], residual=residual)

    # ---- building blocks -------------------------------------------------------------
    def linear(self, name, x, out=None):
        p = self._proj[name]
        if self._tp is not None and name in ('self_attn.o_proj.weight', 'mlp.down_proj.weight'):
            return self._row_parallel(name, x)
        return rt.linear(x, p['fmt'], p['group'], p['n'], p['codes'], p['scales'], down=p['down'], up=p['up'], out=out)

    def _row_parallel(self, name, x, z=None, buf=None):
        """Row-parallel projection: the local partial y_r = half(x_r W_r^T) and the partial
        correction projection z_r = half(x_r V_r^T) share one buffer, one NCCL all-reduce
        (sum) combines both, then y = half(y + half(z U^T)) -- at decode sizes in one GEMV
        launch (the sum as its residual).  ``buf`` / ``z`` (a [M, _ZP] view at its end): the
        buffer and a projection a producer kernel already wrote there (lb_silu_mul_project)."""
        p = self._proj[name]
        m, n = x.shape[0], p['n']
        corr = self._row_corr.get(name)
        if buf is None:
            buf = torch.empty(m * n + (m * _ZP if corr else 0), dtype=torch.float16, device=x.device)
        y = buf[:m * n].view(m, n)
        rt.linear(x, p['fmt'], p['group'], n, p['codes'], p['scales'], out=y)
        if corr is None:
            _all_reduce(buf, self._tp)
            return y
        down, upp = corr
        zv = buf[m * n:].view(m, _ZP)
        if z is None:
            rt.linear(x, 'fp16', x.shape[1], _ZP, down.view(torch.uint8).reshape(-1), None, out=zv)
        _all_reduce(buf, self._tp)
        ucodes = upp.view(torch.uint8).reshape(-1)
        if rt.linear_select('fp16', _ZP, m, n, _ZP) == 'gemv':
            return rt.linear_stacked(zv, 'fp16', _ZP, n, ucodes, None, residual=y)
        delta = rt.linear(zv, 'fp16', _ZP, n, ucodes, None)
        out = torch.empty_like(y)
        rt.check(rt.lib().lb_add(rt.ptr(y), rt.ptr(delta), rt.ptr(out), out.numel(), rt.stream_ptr(x.device)), 'lb_add')
        return out

    def norm(self, x, name, residual=None, residual_out=None, out=None):
        """RMSNorm of x (or of half(x + residual), written to residual_out)."""
        rows, d = x.shape
        out = torch.empty_like(x) if out is None else out
        rt.check(rt.lib().lb_rmsnorm(rt.ptr(x), rt.ptr(residual), rt.ptr(residual_out), rt.ptr(self._norm[name]),
                                     rt.ptr(out), rows, d, self.config.eps, rt.stream_ptr(x.device)), 'lb_rmsnorm')
        return out

    def _attention_prefill(self, q, k, v, b, s):
        """Causal GQA attention for a whole prompt (PyTorch SDPA on the device)."""
        cfg = self.config
        q = q.view(b, s, cfg.heads, cfg.head_dim).transpose(1, 2)
        k = k.view(b, s, cfg.kv_heads, cfg.head_dim).transpose(1, 2)
        v = v.view(b, s, cfg.kv_heads, cfg.head_dim).transpose(1, 2)
        out = F.scaled_dot_product_attention(q, k, v, is_causal=True, scale=1.0 / cfg.head_dim ** 0.5,
                                             enable_gqa=cfg.heads != cfg.kv_heads)
        return out.transpose(1, 2).reshape(b * s, cfg.heads * cfg.head_dim)

    def _qkv(self, normed, positions, rope):
        """q, k, v after RoPE (row views of one buffer when the stacked launch ran)."""
        qkv = self._stacked('qkv', normed)
        if qkv is not None:
            nq, nk, _ = self._stacks['qkv']['widths']
            q, k, v = qkv[:, :nq], qkv[:, nq:nq + nk], qkv[:, nq + nk:]
        else:
            q = self.linear('self_attn.q_proj.weight', normed)
            k = self.linear('self_attn.k_proj.weight', normed)
            v = self.linear('self_attn.v_proj.weight', normed)
        cfg = self.config
        cos, sin = rope
        rt.check(rt.lib().lb_rope(rt.ptr(q), rt.ptr(k), rt.ptr(positions), rt.ptr(cos), rt.ptr(sin), cos.shape[0], q.shape[0],
                                  cfg.heads, cfg.kv_heads, cfg.head_dim, q.stride(0), k.stride(0), rt.stream_ptr(q.device)),
                 'lb_rope')
        return q, k, v

    def _ffn(self, normed, residual=None):
        """down(silu(gate) * up); with ``residual`` the stacked path returns
        half(residual + down) from the down projection's epilogue, else None is returned
        as the second value and the caller adds."""
        gu = self._stacked('gate_up', normed)
        if gu is not None:
            ni = self._stacks['gate_up']['widths'][0]
            gate, up = gu[:, :ni], gu[:, ni:]
        else:
            gate = self.linear('mlp.gate_proj.weight', normed)
            up = self.linear('mlp.up_proj.weight', normed)
        rows, cols = gate.shape
        act = torch.empty(rows, cols, dtype=torch.float16, device=gate.device)
        rt.check(rt.lib().lb_silu_mul(rt.ptr(gate), rt.ptr(up), gate.stride(0), rt.ptr(act), rows, cols,
                                      rt.stream_ptr(gate.device)), 'lb_silu_mul')
        name = 'mlp.down_proj.weight'
        p = self._proj[name]
        if residual is not None and self._tp is None and \
                rt.linear_select(p['fmt'], p['group'], rows, p['n'], p['k']) == 'gemv':
            out = rt.linear_stacked(act, p['fmt'], p['group'], p['n'], p['codes'], p['scales'], down=p['down'],
                                    up=p['up'], residual=residual)
            return out, True
        return self.linear(name, act), False

    def _check_input(self, x):
        if self.training:
            raise ValueError('FrozenSmolLayer requires eval; training is unsupported')
        if (not isinstance(x, torch.Tensor) or x.dtype != torch.float16 or x.ndim != 3 or x.shape[2] != self.config.hidden
                or x.device != self.device):
            raise ValueError(f'Requires FP16 (B,S,{self.config.hidden}) input on {self.device}')

    def _rope(self):
        cache = getattr(self, '_rope_cache', None)
        if cache is None:
            cache = rope_tables(self.config, self.max_positions, self.device)
            self._rope_cache = cache
        return cache

    def _full(self, x):
        b, s, d = x.shape
        h = x.reshape(b * s, d).contiguous()
        pos = torch.arange(s, device=self.device, dtype=torch.int32).repeat(b)
        normed = self.norm(h, 'input_layernorm.weight')
        q, k, v = self._qkv(normed, pos, self._rope())
        attn = self._attention_prefill(q, k, v, b, s)
        o = self.linear('self_attn.o_proj.weight', attn)
        h1 = torch.empty_like(h)
        normed = self.norm(o, 'post_attention_layernorm.weight', residual=h, residual_out=h1)
        down, _ = self._ffn(normed)
        out = torch.empty_like(h)
        rt.check(rt.lib().lb_add(rt.ptr(h1), rt.ptr(down), rt.ptr(out), out.numel(), rt.stream_ptr(out.device)), 'lb_add')
        return out.view(b, s, d), k, v

    # ---- public API (torch_npu_smollm.py:449-544) -------------------------------------
    def forward(self, x):
        self._check_input(x)
        return self._full(x)[0]

    def prefill(self, x):
        """Full prefix; returns the output and a KV snapshot of the prompt."""
        self._check_input(x)
        b, s, _ = x.shape
        out, k, v = self._full(x)
        cfg = self.config
        keys = torch.zeros(b, cfg.kv_heads, self.max_positions, cfg.head_dim, dtype=torch.float16, device=self.device)
        values = torch.zeros_like(keys)
        keys[:, :, :s] = k.view(b, s, cfg.kv_heads, cfg.head_dim).transpose(1, 2)
        values[:, :, :s] = v.view(b, s, cfg.kv_heads, cfg.head_dim).transpose(1, 2)
        return out, SmolKVCache(self._owner, object(), _CacheStore(keys, values, s), s)

    def prefill_into(self, x, keys, values):
        """Prefill writing K/V for positions [0, S) into caller buffers [B, kv_heads, max_pos, hd]."""
        self._check_input(x)
        b, s, _ = x.shape
        out, k, v = self._full(x)
        cfg = self.config
        keys[:, :, :s] = k.view(b, s, cfg.kv_heads, cfg.head_dim).transpose(1, 2)
        values[:, :, :s] = v.view(b, s, cfg.kv_heads, cfg.head_dim).transpose(1, 2)
        return out

    def decode(self, x, cache):
        """Append exactly one token, leaving the previous snapshot valid."""
        self._check_input(x)
        if x.shape[1] != 1 or type(cache) is not SmolKVCache or cache._owner is not self._owner:
            raise ValueError('Decode requires one token and this layer\'s own KV cache')
        if not 1 <= cache.length < self.max_positions:
            raise ValueError('KV cache is full or has an invalid length')
        store = cache._store
        if store.written > cache.length:       # decoding from an older snapshot: copy on write
            store = _CacheStore(store.keys.clone(), store.values.clone(), cache.length)
        b = x.shape[0]
        lengths = torch.full((b,), cache.length, dtype=torch.int32, device=self.device)
        h = x.reshape(b, -1).contiguous()
        out = self.decode_step(h, store.keys, store.values, lengths)
        store.written = cache.length + 1
        return out.view(b, 1, -1), SmolKVCache(self._owner, cache._sequence, store, cache.length + 1)

    def decode_step(self, h, k_cache, v_cache, lengths, normed=None):
        """One token for every sequence: h [B, d] -> output [B, d]; writes K/V at lengths[b].

        Decode batches (<= 64 rows) run 9 launches per layer: RMSNorm + z(q|k|v), the
        stacked q|k|v GEMV, RoPE + KV append + attention, z(o) + o GEMV, RMSNorm with the
        residual + z(gate|up), the stacked gate|up GEMV, SiLU-mul + z(down), and the down
        GEMV with the residual add in its epilogue."""
        cfg = self.config
        b = h.shape[0]
        L = rt.lib()
        st = rt.stream_ptr(h.device)
        qs = self._stack_for('qkv', b)
        # z fused into the row producers only for small batches: from 16 rows on, the
        # projection kernel that shares each V row across 8 activation rows is faster
        fuse_z = b <= _FUSE_Z_ROWS
        z = None
        if normed is None:
            normed, z = self._norm_project(h, 'input_layernorm.weight',
                                           None if qs is None or not fuse_z else qs['down'])
        if qs is not None:
            qkv = rt.linear_stacked(normed, qs['fmt'], qs['group'], qs['n'], qs['codes'], qs['scales'],
                                    down=qs['down'] if z is None else None, up=qs['up'], z=z)
            nq, nk, _ = qs['widths']
            q, k, v = qkv[:, :nq], qkv[:, nq:nq + nk], qkv[:, nq + nk:]
        else:
            q = self.linear('self_attn.q_proj.weight', normed)
            k = self.linear('self_attn.k_proj.weight', normed)
            v = self.linear('self_attn.v_proj.weight', normed)
        cos, sin = self._rope()
        attn = torch.empty(b, cfg.heads * cfg.head_dim, dtype=torch.float16, device=h.device)
        # RoPE of q / k at lengths[b], KV append and attention in one launch
        # the stream's linear workspace also holds the attention's position-split scratch
        ws = rt.Workspace.get(L.lb_attention_workspace_bytes(b, cfg.heads, self.max_positions), h.device)
        rt.check(L.lb_attention_decode_rope(rt.ptr(q), q.stride(0), rt.ptr(k), rt.ptr(v), k.stride(0), rt.ptr(cos),
                                            rt.ptr(sin), cos.shape[0], rt.ptr(k_cache), rt.ptr(v_cache), rt.ptr(lengths),
                                            rt.ptr(attn), b, cfg.heads, cfg.kv_heads, cfg.head_dim, self.max_positions,
                                            1.0 / cfg.head_dim ** 0.5, rt.ptr(ws), ws.numel(), st),
                 'lb_attention_decode_rope')
        o = self.linear('self_attn.o_proj.weight', attn)
        h1 = torch.empty_like(h)
        gs = self._stack_for('gate_up', b)
        normed, z = self._norm_project(o, 'post_attention_layernorm.weight',
                                       None if gs is None or not fuse_z else gs['down'], residual=h, residual_out=h1)
        if gs is not None:
            gu = rt.linear_stacked(normed, gs['fmt'], gs['group'], gs['n'], gs['codes'], gs['scales'],
                                   down=gs['down'] if z is None else None, up=gs['up'], z=z)
            ni = gs['widths'][0]
            gate, up = gu[:, :ni], gu[:, ni:]
        else:
            gate = self.linear('mlp.gate_proj.weight', normed)
            up = self.linear('mlp.up_proj.weight', normed)
        dp = self._proj['mlp.down_proj.weight']
        fused_down = self._tp is None and rt.linear_select(dp['fmt'], dp['group'], b, dp['n'], dp['k']) == 'gemv'
        rows, cols = gate.shape
        act = torch.empty(rows, cols, dtype=torch.float16, device=h.device)
        if self._tp is not None:
            # row-parallel down projection: SiLU-mul writes the partial z = act . V_r^T
            # straight into the buffer the all-reduce sums
            corr = self._row_corr.get('mlp.down_proj.weight')
            buf = torch.empty(rows * dp['n'] + (rows * _ZP if corr else 0), dtype=torch.float16, device=h.device)
            zv = buf[rows * dp['n']:].view(rows, _ZP) if corr else None
            rt.check(L.lb_silu_mul_project(rt.ptr(gate), rt.ptr(up), gate.stride(0), rt.ptr(act), rows, cols,
                                           rt.ptr(corr[0] if corr else None), _ZP if corr else 0, rt.ptr(zv), st),
                     'lb_silu_mul_project')
            down = self._row_parallel('mlp.down_proj.weight', act, z=zv, buf=buf)
            out = torch.empty_like(h)
            rt.check(L.lb_add(rt.ptr(h1), rt.ptr(down), rt.ptr(out), out.numel(), st), 'lb_add')
            return out
        zd = None
        if fused_down and fuse_z and dp['down'] is not None:
            zd = torch.empty(rows, (dp['down'].shape[0] + 31) // 32 * 32, dtype=torch.float16, device=h.device)
        rt.check(L.lb_silu_mul_project(rt.ptr(gate), rt.ptr(up), gate.stride(0), rt.ptr(act), rows, cols,
                                       rt.ptr(dp['down'] if zd is not None else None),
                                       0 if zd is None else dp['down'].shape[0], rt.ptr(zd), st), 'lb_silu_mul_project')
        if fused_down:
            return rt.linear_stacked(act, dp['fmt'], dp['group'], dp['n'], dp['codes'], dp['scales'],
                                     down=dp['down'] if zd is None else None, up=dp['up'], z=zd, residual=h1)
        down = self.linear('mlp.down_proj.weight', act)
        out = torch.empty_like(h)
        rt.check(L.lb_add(rt.ptr(h1), rt.ptr(down), rt.ptr(out), out.numel(), st), 'lb_add')
        return out

    def _stack_for(self, key, rows):
        """The stacked projection when its single decode-GEMV launch applies, else None."""
        st = self._stacks.get(key)
        if st is None or rt.linear_select(st['fmt'], st['group'], rows, st['n'], st['k']) != 'gemv':
            return None
        return st

    def _norm_project(self, x, name, down, residual=None, residual_out=None):
        """RMSNorm (+ residual) of x and, when ``down`` is given, z = half(normed . down^T)
        for the linear that reads it (lb_rmsnorm_project): (normed, z or None)."""
        rows, d = x.shape
        out = torch.empty(rows, d, dtype=torch.float16, device=x.device)
        z = None
        if down is not None:
            z = torch.empty(rows, (down.shape[0] + 31) // 32 * 32, dtype=torch.float16, device=x.device)
        rt.check(rt.lib().lb_rmsnorm_project(rt.ptr(x), rt.ptr(residual), rt.ptr(residual_out), rt.ptr(self._norm[name]),
                                             rt.ptr(out), rows, d, self.config.eps, rt.ptr(down),
                                             0 if down is None else down.shape[0], rt.ptr(z), rt.stream_ptr(x.device)),
                 'lb_rmsnorm_project')
        return out, z


class FrozenSmolStack(torch.nn.Module):
    """Contiguous decoder layers (torch_npu_smollm.py:558-657).

    ``FrozenSmolStack(directory, *, start_layer, num_layers, mode, packed_weights,
    fp16_projections, corrections)`` loads the layer range of a SmolLM safetensors
    checkpoint directory as the reference does, with the same validation; the GPU
    keywords ``group_size``, ``device`` and ``max_positions`` are passed to every layer.
    ``packed_weights`` / ``corrections`` are maps indexed by checkpoint layer, e.g. as
    read by torch_npu_lowbit_checkpoint.load_packed.  Corrections are accepted for every
    quantized mode (the reference: W8 with explicit packed weights only).
    ``FrozenSmolStack.from_layers(layers)`` wraps layers built in memory (no reference
    counterpart).
    """

    def __init__(self, directory, *, start_layer=0, num_layers=2, mode='w8a16', packed_weights=None,
                 fp16_projections=(), corrections=None, group_size=None, device=None, max_positions=None):
        super().__init__()
        self._fp16_projections = _projection_policy(mode, fp16_projections)
        directory = Path(directory)
        config = json.loads((directory / 'config.json').read_text())
        total = config.get('num_hidden_layers', 0)
        if (type(start_layer) is not int or type(num_layers) is not int or type(total) is not int
                or start_layer < 0 or num_layers <= 0 or start_layer + num_layers > total):
            raise ValueError('Requires a nonempty contiguous checkpoint layer range')
        if mode not in _WEIGHT_FORMATS:
            raise ValueError('Requires fp16, w8a16, w4a16 or nf4a16')
        indices = set(range(start_layer, start_layer + num_layers))
        if packed_weights is not None and (mode == 'fp16' or type(packed_weights) is not dict
                                           or any(type(i) is not int for i in packed_weights)
                                           or any(type(v) is not dict for v in packed_weights.values())
                                           or set(packed_weights) != indices):
            raise ValueError('Prepared stack weights require a complete lowbit map indexed by checkpoint layer')
        if corrections is not None and (mode == 'fp16' or type(corrections) is not dict
                                        or any(type(i) is not int or type(v) is not dict for i, v in corrections.items())
                                        or set(corrections) != indices):
            raise ValueError('Stack corrections require a quantized mode and a complete map indexed by checkpoint layer')
        from safetensors import safe_open
        layers = []
        with safe_open(directory / 'model.safetensors', framework='pt', device='cpu') as file:
            names = list(file.keys())
            for i in range(start_layer, start_layer + num_layers):
                prefix = f'model.layers.{i}.'
                weights = {n[len(prefix):]: file.get_tensor(n) for n in names if n.startswith(prefix)}
                layers.append(FrozenSmolLayer(config, weights, mode=mode,
                                              packed_weights=None if packed_weights is None else packed_weights[i],
                                              fp16_projections=fp16_projections,
                                              corrections=None if corrections is None else corrections[i],
                                              group_size=group_size, device=device, max_positions=max_positions))
        self._set_layers(layers, start_layer, mode)

    def _set_layers(self, layers, start_layer, mode):
        self.layers = torch.nn.ModuleList(layers)
        self.start_layer = start_layer
        self._mode = mode
        self.eval()

    @classmethod
    def from_layers(cls, layers, *, start_layer=0):
        """A stack of layers already built in memory."""
        if not layers or any(not isinstance(l, FrozenSmolLayer) for l in layers):
            raise ValueError('Requires a nonempty list of FrozenSmolLayer')
        self = cls.__new__(cls)
        torch.nn.Module.__init__(self)
        self._fp16_projections = layers[0].fp16_projections
        self._set_layers(layers, start_layer, layers[0].mode)
        return self

    @classmethod
    def from_checkpoint(cls, directory, **options):
        return cls(directory, **options)

    mode = property(lambda self: self._mode)
    fp16_projections = property(lambda self: self._fp16_projections)

    def reference_cpu(self, x, *, quantized=True):
        """Not provided (see FrozenSmolLayer.reference_cpu)."""
        raise NotImplementedError('reference_cpu is the CPU test oracle; this package runs on the GPU only')

    @property
    def num_layers(self):
        return len(self.layers)

    def forward(self, x):
        for layer in self.layers:
            x = layer(x)
        return x

    def prefill(self, x):
        caches, sequence = [], object()
        for layer in self.layers:
            x, cache = layer.prefill(x)
            caches.append(SmolKVCache(cache._owner, sequence, cache._store, cache.length))
        return x, tuple(caches)

    def decode(self, x, caches, *, group_size=None):
        """group_size is the reference's NPU chain width (1, 2 or 4); accepted and validated only."""
        if group_size is not None and group_size not in (1, 2, 4):
            raise ValueError('Decode group_size must be 1, 2 or 4')
        if type(caches) is not tuple or len(caches) != self.num_layers:
            raise ValueError('Requires one KV cache per consecutive layer')
        if any(c.length != caches[0].length or c._sequence is not caches[0]._sequence for c in caches):
            raise ValueError('Stack KV caches must belong to the same snapshot and position')
        updated, sequence = [], object()
        for layer, cache in zip(self.layers, caches):
            x, cache = layer.decode(x, cache)
            updated.append(SmolKVCache(cache._owner, sequence, cache._store, cache.length))
        return x, tuple(updated)


class SmolForCausalLM(torch.nn.Module):
    """Decoder stack + tied fp16 embedding / LM head (FrozenSmolIO) with greedy generation.

    The decode step (all layers + head + argmax) is captured once per batch size in a
    CUDA graph and replayed per token.  No reference counterpart: the reference drives its
    stack and FrozenSmolIO from the caller (torch_npu_smollm_io.py:14-61).
    """

    def __init__(self, stack, embedding, norm):
        super().__init__()
        self.stack = stack
        self.config = stack.layers[0].config
        self.device = stack.layers[0].device
        cfg = dict(model_type='llama', hidden_size=self.config.hidden, vocab_size=self.config.vocab,
                   tie_word_embeddings=True, rms_norm_eps=self.config.eps)
        self.io = FrozenSmolIO(cfg, embedding, norm, device=self.device)
        self.embedding = self.io.embedding
        self.final_norm = self.io.norm
        self._graphs = {}
        # tensor-parallel stacks keep their all-reduces out of the captured graphs: NCCL
        # all-reduces captured in the decode-step graph gave wrong logits (and, in one harness,
        # never completed) on B200 + NCCL 2.28, so the step is graphs split at the all-reduces
        self._tensor_parallel = any(l._tp is not None for l in stack.layers)

    @classmethod
    def from_weights(cls, config, layer_weights, embedding, norm, **layer_options):
        layers = [FrozenSmolLayer(config, w, **layer_options) for w in layer_weights]
        return cls(FrozenSmolStack.from_layers(layers), embedding, norm)

    @classmethod
    def from_checkpoint(cls, directory, **stack_options):
        """Every layer of a SmolLM checkpoint directory plus its tied endpoints; the options
        are FrozenSmolStack's (mode, packed_weights, corrections, group_size, ...)."""
        from safetensors import safe_open
        directory = Path(directory)
        total = json.loads((directory / 'config.json').read_text()).get('num_hidden_layers', 0)
        stack = FrozenSmolStack(directory, start_layer=0, num_layers=total, **stack_options)
        with safe_open(directory / 'model.safetensors', framework='pt', device='cpu') as f:
            emb, norm = f.get_tensor('model.embed_tokens.weight'), f.get_tensor('model.norm.weight')
        return cls(stack, emb, norm)

    def embed(self, ids):
        return self.io.embed_rows(ids)

    def head(self, h, residual=None):
        """Final RMSNorm (fused with the last residual add) + tied LM head -> fp16 logits."""
        return self.io.head_rows(h, residual)

    def argmax(self, logits, out):
        rt.check(rt.lib().lb_argmax(rt.ptr(logits), logits.shape[0], logits.shape[1], rt.ptr(out), None, 0,
                                    rt.stream_ptr(self.device)), 'lb_argmax')
        return out

    def prefill(self, ids):
        """ids [B, S] int64 on the device -> (last-position logits [B, V], caches)."""
        b, s = ids.shape
        x = self.embed(ids.reshape(-1)).view(b, s, -1)
        h, caches = self.stack.prefill(x)
        last = h[:, -1].contiguous()
        return self.head(last), caches

    def session(self, b):
        """Device state for batch size b, allocated once and reused: token ids, per-sequence
        lengths, per-layer KV caches [b, kv_heads, max_pos, hd] and the captured decode graph."""
        st = self._graphs.get(b)
        if st is None:
            cfg, layers = self.config, self.stack.layers
            mp = layers[0].max_positions
            st = dict(
                ids=torch.zeros(b, dtype=torch.int64, device=self.device),
                lengths=torch.zeros(b, dtype=torch.int32, device=self.device),
                keys=[torch.zeros(b, l.config.kv_heads, mp, cfg.head_dim, dtype=torch.float16, device=self.device)
                      for l in layers],
                values=[torch.zeros(b, l.config.kv_heads, mp, cfg.head_dim, dtype=torch.float16, device=self.device)
                        for l in layers],
                graph=None, logits=None)
            self._graphs[b] = st
        return st

    def prefill_session(self, ids):
        """Prefill ``ids`` [B, S] into the batch's session: caches filled for [0, S), lengths
        set to S, ids set to the greedy next token.  Returns the last-position logits."""
        b, s = ids.shape
        st = self.session(b)
        x = self.embed(ids.reshape(-1)).view(b, s, -1)
        for i, layer in enumerate(self.stack.layers):
            x = layer.prefill_into(x, st['keys'][i], st['values'][i])
        logits = self.head(x[:, -1].contiguous())
        st['lengths'].fill_(s)
        self.argmax(logits, st['ids'])
        return logits

    def _decode_step(self, st):
        """Embed st['ids'], run every layer at positions st['lengths'], write logits and the
        greedy next ids, advance the lengths."""
        h = self.embed(st['ids'])
        for i, layer in enumerate(self.stack.layers):
            h = layer.decode_step(h, st['keys'][i], st['values'][i], st['lengths'])
        logits = self.head(h)
        self.argmax(logits, st['ids'])
        st['lengths'] += 1
        return logits

    def decode_step(self, b, graph=True):
        """One greedy token for every sequence of the batch's session; returns fp16 logits.
        The step is a replayed CUDA graph; for a tensor-parallel stack, a chain of graphs split
        at its all-reduces, which run eagerly between them (_PiecewiseGraph)."""
        st = self.session(b)
        if not graph:
            return self._decode_step(st)
        if self._tensor_parallel:
            if st.get('piecewise') is None:
                self._capture(st, piecewise=True)
            st['piecewise'].replay()
            return st['logits']
        if st['graph'] is None:
            self._capture(st)
        st['graph'].replay()
        return st['logits']

    def _capture(self, st, piecewise=False):
        stream = torch.cuda.current_stream(self.device)
        saved, ids = st['lengths'].clone(), st['ids'].clone()
        side = torch.cuda.Stream(self.device)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            self._decode_step(st)            # warm-up: sizes workspaces outside capture
            st['lengths'].copy_(saved)
            st['ids'].copy_(ids)
            if piecewise:
                side.synchronize()
                rec = _PiecewiseGraph()
                st['logits'] = rec.record(lambda: self._decode_step(st))
            else:
                g = torch.cuda.CUDAGraph(keep_graph=True)   # kept for launch counting (cudaGraphGetNodes)
                with torch.cuda.graph(g, stream=side):
                    st['logits'] = self._decode_step(st)
        stream.wait_stream(side)
        if piecewise:
            st['piecewise'] = rec
        else:
            st['graph'] = g

    def generate(self, ids, steps, *, graph=True, return_logits=False):
        """Greedy decoding: prefill ``ids`` [B, S] (device int64), then ``steps`` tokens.

        Returns next tokens [B, steps] (and the fp16 logits of each step when asked)."""
        b, s = ids.shape
        if s + steps > self.stack.layers[0].max_positions:
            raise ValueError('prompt + generated tokens exceed max_positions of the KV cache')
        st = self.session(b)
        logits = self.prefill_session(ids)
        tokens = torch.empty(b, steps, dtype=torch.int64, device=self.device)
        all_logits = [logits.clone()] if return_logits else None
        tokens[:, 0] = st['ids']
        for t in range(1, steps):
            out = self.decode_step(b, graph=graph)
            tokens[:, t] = st['ids']
            if return_logits:
                all_logits.append(out.clone())
        # a bounded device-side wait that ran out inside a replayed step is reported here
        # (one synchronising read of each workspace status word)
        rt.check_device_waits(self.device)
        return (tokens, all_logits) if return_logits else tokens


def random_smollm_weights(config, seed=0, device='cpu', std=0.02):
    """Random-init SmolLM weights (std 0.02, unit norms) for synthetic benchmarks and tests."""
    cfg = config if isinstance(config, SmolConfig) else SmolConfig.from_dict(config)
    gen = torch.Generator(device=device).manual_seed(seed)
    layers = []
    for _ in range(cfg.layers):
        w = {}
        for name, shape in cfg.shapes().items():
            if len(shape) == 2:
                w[name] = (torch.randn(shape, generator=gen, device=device) * std).half()
            else:
                w[name] = torch.ones(shape, dtype=torch.float16, device=device)
        layers.append(w)
    embedding = (torch.randn(cfg.vocab, cfg.hidden, generator=gen, device=device) * std).half()
    norm = torch.ones(cfg.hidden, dtype=torch.float16, device=device)
    return layers, embedding, norm
