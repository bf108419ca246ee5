"""On-disk packed low-bit weights: one safetensors file of codes, scales and correction
factors, loaded straight to the GPU.

The reference keeps nothing of the quantized model on disk except compiled NPU graph
blobs (torch_npu_graph_cache.py:102-134, opt-in through NPUNLOCK_GRAPH_CACHE): every
start re-reads fp16 safetensors (torch_npu_smollm.py:120-127, :584-590) and quantizes.
Here the packed model itself is the cache: the canonical packed bytes of every
projection (pack_codes order, torch_npu_lowbit.py:24-30), its fp16 scales and its
LowRankCorrection factors, keyed by checkpoint layer, so that a start skips quantization
and the bytes go from the file to HBM without a host-side repack.

File layout (safetensors, little-endian):
  model.layers.<i>.<projection>.codes   uint8  [packed bytes]
  model.layers.<i>.<projection>.scales  fp16   [N * K / group]
  model.layers.<i>.<projection>.down    fp16   [rank, K]   (when the layer has a correction)
  model.layers.<i>.<projection>.up      fp16   [N, rank]
and the metadata header: ``lowbit_packed`` = format version, and for every projection
``model.layers.<i>.<projection>`` = JSON {"shape": [N, K], "format": ..., "group_size": ...}.
"""
import json
from pathlib import Path

import numpy as np
import torch

from torch_npu_lowbit import DevicePackedWeight, PackedWeight
from torch_npu_lowbit_correction import LowRankCorrection

VERSION = '1'


def save_packed(path, packed_weights, corrections=None):
    """Write ``packed_weights`` {layer: {projection: PackedWeight | DevicePackedWeight}} and
    optional ``corrections`` {layer: {projection: LowRankCorrection}} to ``path``."""
    from safetensors.torch import save_file
    if type(packed_weights) is not dict or not packed_weights:
        raise ValueError('Packed checkpoint requires a nonempty map indexed by checkpoint layer')
    tensors, meta = {}, {'lowbit_packed': VERSION}
    for layer, projections in packed_weights.items():
        if type(layer) is not int or type(projections) is not dict:
            raise ValueError('Packed checkpoint requires a map indexed by checkpoint layer')
        for name, q in projections.items():
            if isinstance(q, DevicePackedWeight):
                q = q.to_host()
            if not isinstance(q, PackedWeight):
                raise ValueError('Packed checkpoint entries must be PackedWeight')
            key = f'model.layers.{layer}.{name}'
            tensors[key + '.codes'] = torch.frombuffer(bytearray(q.data), dtype=torch.uint8)
            tensors[key + '.scales'] = torch.frombuffer(bytearray(q.scales), dtype=torch.float16)
            meta[key] = json.dumps({'shape': list(q.shape), 'format': q.format, 'group_size': q.group_size})
    for layer, projections in (corrections or {}).items():
        for name, c in projections.items():
            key = f'model.layers.{layer}.{name}'
            if key not in meta or not isinstance(c, LowRankCorrection):
                raise ValueError('A correction needs a LowRankCorrection on a packed projection')
            down, up = c.tensors()
            tensors[key + '.down'], tensors[key + '.up'] = down, up
    save_file(tensors, str(path), metadata=meta)


def load_packed(path, *, device=None):
    """Read a packed checkpoint: (packed_weights, corrections), both indexed by checkpoint
    layer.  With ``device`` the codes and scales are loaded straight to that CUDA device as
    DevicePackedWeight; without it they are host PackedWeight (validated as the
    reference validates them).  Corrections are LowRankCorrection (host bytes)."""
    from safetensors import safe_open
    path = Path(path)
    target = 'cpu' if device is None else str(torch.device(device))
    packed, corrections = {}, {}
    with safe_open(str(path), framework='pt', device='cpu') as f:
        meta = f.metadata() or {}
        if meta.get('lowbit_packed') != VERSION:
            raise ValueError('Not a low-bit packed checkpoint of a supported version')
        entries = {k: json.loads(v) for k, v in meta.items() if k.startswith('model.layers.')}
        factors = {}
        for key in entries:
            if key + '.down' in f.keys():
                factors[key] = (f.get_tensor(key + '.down'), f.get_tensor(key + '.up'))
    with safe_open(str(path), framework='pt', device=target) as f:
        for key, e in entries.items():
            _, _, layer, name = key.split('.', 3)
            layer = int(layer)
            shape = tuple(int(v) for v in e['shape'])
            codes, scales = f.get_tensor(key + '.codes'), f.get_tensor(key + '.scales')
            if device is None:
                q = PackedWeight(shape, e['format'], int(e['group_size']), codes.numpy().tobytes(),
                                 scales.numpy().tobytes())
            else:
                q = DevicePackedWeight(shape, e['format'], int(e['group_size']), codes, scales)
            packed.setdefault(layer, {})[name] = q
            if key in factors:
                down, up = factors[key]
                corrections.setdefault(layer, {})[name] = LowRankCorrection(
                    shape, down.shape[0], np.ascontiguousarray(down.numpy()).tobytes(),
                    np.ascontiguousarray(up.numpy()).tobytes())
    return packed, (corrections or None)
