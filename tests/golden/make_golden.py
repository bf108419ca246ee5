"""Generate the golden fixtures that pin the oracle to the reference implementation.

Run in a container where the reference checkout is importable, e.g.::

    REF=/path/to/torch-intel-npu python tests/golden/make_golden.py

It imports the reference's own CPU code (torch_npu_lowbit, torch_npu_lowbit_correction,
torch_npu_smollm, torch_npu_smollm_io), runs it on seeded synthetic inputs and writes
small ``.npz`` fixtures next to this script.  Tests never import the reference; they
compare the oracle (and, on a GPU, the CUDA path) against these files.
Large weights are not stored: the fixture records the seed plus a SHA-256 of the
regenerated weights, so a test can rebuild them and detect RNG drift.
"""
import hashlib
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
if not os.environ.get('REF'):
    sys.exit('set REF to the reference checkout (the directory holding torch_npu_lowbit.py)')
REF = Path(os.environ['REF'])
sys.path[:0] = [str(REF), str(REF / 'npunlock/python')]

import torch_npu_lowbit as lb  # noqa: E402
import torch_npu_lowbit_correction as lc  # noqa: E402

# The reference bounds N*K by an NPU storage limit (npunlock/npu4000.py:23); lift it
# for the B200 shapes exactly as the reference's own module global allows.
lb.MAX_TENSOR_ELEMENTS = 1 << 26
lc.MAX_TENSOR_ELEMENTS = 1 << 26


def sha(b):
    return hashlib.sha256(b).hexdigest()


def tensor_sha(t):
    return sha(t.detach().contiguous().numpy().tobytes())


# ---------------------------------------------------------------------------------
# 1. quantize/pack + dequantize on seeded and adversarial weights
# ---------------------------------------------------------------------------------
def adversarial(fmt, group):
    """Weights that sit on every rounding decision the quantizer makes."""
    rows = []
    g = group
    # exact .5 ties for the integer formats and exact NF4 midpoints, at scale 1
    if fmt == 'nf4':
        mids = (lb.NF4[:-1] + lb.NF4[1:]) / 2
        base = np.concatenate((mids, lb.NF4, np.nextafter(mids, np.float32(2)), np.nextafter(mids, np.float32(-2))))
    else:
        limit = 7 if fmt == 'int4' else 127
        base = np.arange(-limit, limit + 1, dtype=np.float32)
        base = np.concatenate((base, base + np.float32(.5), base - np.float32(.5)))
        base = np.clip(base, -limit, limit)
    row = np.resize(base.astype(np.float32), g)
    row[0] = 1.0 if fmt == 'nf4' else float(7 if fmt == 'int4' else 127)   # pin absmax -> scale 1
    rows.append(row)
    rows.append(-row)
    rows.append(np.zeros(g, np.float32))                      # zero group -> 2^-24 scale
    tiny = np.resize(np.array([3e-8, -1e-7, 2e-9, 5e-8], np.float32), g)
    rows.append(tiny)                                         # subnormal fp16 scales
    rows.append(np.resize(np.array([60000., -1., .5, 1e-3], np.float32), g))  # large dynamic range
    return np.stack(rows)


def quant_cases():
    gen = torch.Generator().manual_seed(0)
    cases = []
    for (n, k) in ((3, 17), (8, 64), (4, 128), (5, 9), (4, 576), (2, 1536), (3, 960), (2, 2560)):
        w32 = torch.randn(n, k, generator=gen) * 0.02
        for dtype in (torch.float32, torch.float16):
            w = w32.to(dtype)
            for fmt in ('int4', 'nf4', 'int8'):
                groups = [None] + [g for g in (3, 32, 64, 128) if k % g == 0 and g < k]
                for g in groups:
                    cases.append((f'rand_{n}x{k}_{str(dtype)[6:]}', w, fmt, g))
    for fmt in ('int4', 'nf4', 'int8'):
        for g in (64, 128):
            a = torch.from_numpy(adversarial(fmt, g))
            cases.append((f'adv_{fmt}_{g}', a, fmt, g))
            cases.append((f'adv16_{fmt}_{g}', a.half(), fmt, g))
    return cases


def make_quant():
    out = {}
    for wname, w, fmt, g in quant_cases():
        q = lb.quantize_weight(w, format=fmt, group_size=g)
        out[f'{wname}/w'] = w.numpy()
        name = f'{wname}/{fmt}_g{q.group_size}'
        out[f'{name}/data'] = np.frombuffer(q.data, np.uint8)
        out[f'{name}/scales'] = np.frombuffer(q.scales, np.uint16)
        out[f'{name}/deq_sha'] = np.array(sha(q.dequantize().tobytes()))
    # rejections (the error classes the reference raises)
    np.savez_compressed(HERE / 'quantize.npz', **out)
    print('quantize.npz', sum(k.endswith('/data') for k in out), 'cases')


# ---------------------------------------------------------------------------------
# 2. BASELINE config shapes: codes/scales digests at full size (seed 0)
# ---------------------------------------------------------------------------------
def baseline_weight(n, k, seed=0):
    gen = torch.Generator().manual_seed(seed)
    w = (torch.randn(n, k, generator=gen) * 0.02).half()
    u = (torch.randn(n, 32, generator=gen) * 1e-3).half()
    v = (torch.randn(32, k, generator=gen) * 1e-3).half()
    return w, u, v


def make_baseline_digests():
    out = {}
    for (n, k) in ((1536, 576), (576, 1536), (8192, 2048), (2048, 8192)):
        w, u, v = baseline_weight(n, k)
        out[f'{n}x{k}/w_sha'] = np.array(tensor_sha(w))
        for fmt, g in (('int8', None), ('int4', 64), ('int4', 128), ('nf4', 64), ('nf4', 128)):
            if g is not None and k % g:
                continue
            q = lb.quantize_weight(w, format=fmt, group_size=g)
            key = f'{n}x{k}/{fmt}_g{q.group_size}'
            out[key + '/data_sha'] = np.array(sha(q.data))
            out[key + '/scales_sha'] = np.array(sha(q.scales))
            out[key + '/deq_sha'] = np.array(sha(q.dequantize().tobytes()))
    np.savez_compressed(HERE / 'baseline_digests.npz', **out)
    print('baseline_digests.npz', len(out))


# ---------------------------------------------------------------------------------
# 3. SmolLM layer reference_cpu traces (135M dims, theta 1e5, <=64 positions)
# ---------------------------------------------------------------------------------
CONFIG = dict(model_type='llama', hidden_size=576, intermediate_size=1536, num_attention_heads=9,
              num_key_value_heads=3, hidden_act='silu', attention_bias=False, mlp_bias=False,
              rms_norm_eps=1e-5, rope_theta=100000, rope_scaling=None, pretraining_tp=1)
SHAPES = {'self_attn.q_proj.weight': (576, 576), 'self_attn.k_proj.weight': (192, 576),
          'self_attn.v_proj.weight': (192, 576), 'self_attn.o_proj.weight': (576, 576),
          'mlp.gate_proj.weight': (1536, 576), 'mlp.up_proj.weight': (1536, 576),
          'mlp.down_proj.weight': (576, 1536), 'input_layernorm.weight': (576,),
          'post_attention_layernorm.weight': (576,)}
TRACE_KEYS = ('norm1', 'keys', 'values', 'attention', 'attention_output', 'residual1', 'norm2',
              'silu', 'gated', 'ffn_output', 'output')


def layer_weights(seed):
    """Same construction as the reference fixture test_torch_npu_smollm_policy.py:287-290."""
    gen = torch.Generator().manual_seed(seed)
    weights = {name: (torch.randn(shape, generator=gen) * .015).half() if len(shape) == 2 else torch.ones(shape).half()
               for name, shape in SHAPES.items()}
    x = (torch.randn(2, 7, 576, generator=gen) * .1).half()
    return weights, x


def layer_corrections(seed):
    gen = torch.Generator().manual_seed(seed)
    out = {}
    for name, shape in SHAPES.items():
        if len(shape) == 2:
            n, k = shape
            down = (torch.randn(32, k, generator=gen) * 1e-3).half()
            up = (torch.randn(n, 32, generator=gen) * 1e-3).half()
            out[name] = (down, up)
    return out


def make_layer():
    import torch_npu_smollm as sm
    out = {}
    weights, x = layer_weights(414)
    out['weights_sha'] = np.array(sha(b''.join(tensor_sha(weights[k]).encode() for k in sorted(weights))))
    out['x'] = x.numpy().view(np.uint16)
    corr = layer_corrections(415)
    out['corr_sha'] = np.array(sha(b''.join((tensor_sha(a) + tensor_sha(b)).encode() for _, (a, b) in sorted(corr.items()))))
    runs = {}
    # fp16 mode
    runs['fp16'] = sm.FrozenSmolLayer(CONFIG, weights, mode='fp16')
    # W8 per-row + rank-32 corrections on all seven projections
    packed8 = {n: lb.quantize_weight(w, format='int8') for n, w in weights.items() if w.ndim == 2}
    cobj = {n: lc.LowRankCorrection(SHAPES[n], 32, d.numpy().tobytes(), u.numpy().tobytes()) for n, (d, u) in corr.items()}
    runs['w8'] = sm.FrozenSmolLayer(CONFIG, weights, mode='w8a16', packed_weights=packed8)
    runs['w8corr'] = sm.FrozenSmolLayer(CONFIG, weights, mode='w8a16', packed_weights=packed8, corrections=cobj)
    for fmt, mode in (('int4', 'w4a16'), ('nf4', 'nf4a16')):
        for g in (32, 64):
            packed = {n: lb.quantize_weight(w, format=fmt, group_size=g) for n, w in weights.items() if w.ndim == 2}
            runs[f'{fmt}_g{g}'] = sm.FrozenSmolLayer(CONFIG, weights, mode=mode, packed_weights=packed)
    for tag, layer in runs.items():
        y, trace = layer.reference_cpu(x)
        out[f'{tag}/y'] = y.numpy().view(np.uint16)
        for key in TRACE_KEYS:
            out[f'{tag}/{key}'] = trace[key].contiguous().numpy().view(np.uint16)
    np.savez_compressed(HERE / 'smollm_layer.npz', **out)
    print('smollm_layer.npz', len(out))


def make_io():
    import torch_npu_smollm_io as io
    gen = torch.Generator().manual_seed(416)
    vocab = 1024
    emb = (torch.randn(vocab, 576, generator=gen) * 0.02).half()
    norm = (1 + 0.1 * torch.randn(576, generator=gen)).half()
    hidden = torch.randn(2, 3, 576, generator=gen).half()
    ids = torch.randint(0, vocab, (2, 5), generator=gen)
    m = io.FrozenSmolIO(dict(model_type='llama', hidden_size=576, tie_word_embeddings=True, rms_norm_eps=1e-5,
                             vocab_size=vocab), emb, norm)
    out = dict(emb_sha=np.array(tensor_sha(emb)), norm=norm.numpy().view(np.uint16),
               hidden=hidden.numpy().view(np.uint16), ids=ids.numpy(),
               logits=m.logits(hidden).numpy().view(np.uint16),
               embedded=m.embed_tokens(ids).numpy().view(np.uint16))
    np.savez_compressed(HERE / 'smollm_io.npz', **out)
    print('smollm_io.npz')


if __name__ == '__main__':
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    make_quant()
    make_baseline_digests()
    make_layer()
    make_io()
