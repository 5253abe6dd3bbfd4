"""The fp16 inference checkpoint, model_latest_fp16.pt, and its lossless per-level support storage.

Format (the artifact odie/train.py:199-216 writes with torch.save, read back by the reference's evaluate and
scripts/reconstruct.py): a dict with
  version 'packed-capacity-control-v1', configuration, settings, checkpoint 'latest', epoch, optimizer_steps,
  metrics, parameters {parameter name: fp16 CPU tensor} (named_parameters of the model: grid, gate.params,
  decoder.params), support_num_cells [R^2 per level], support_payload (the support record without its masks),
  support_metadata, support_storage_version 'layerwise-bitmap-deflate-jbig-v1' and support_encodings, one
  record per level: num_cells, resolution, selected_count, encoding and (unless constant) data, a flat uint8
  tensor.
Encodings (odie/support_codec.py:51-153): 'all' / 'none' for a constant mask; otherwise the shortest of
'bitmap' (the cells LSB-first, np.packbits little order) and 'bitmap_deflate' (that bitmap as a raw DEFLATE
stream, zlib level 9, window bits -15), the raw bitmap winning ties.  The reference may also pick 'jbig1'
through an optional libjbig command-line bridge; libjbig is not part of this build, so -- exactly as the
reference does when that bridge cannot be built -- masks are written as bitmap / DEFLATE, and a 'jbig1' record
is refused on reading.
"""
import math
from pathlib import Path
import zlib

import numpy as np
import torch

ARTIFACT_VERSION = 'packed-capacity-control-v1'
STORAGE_VERSION = 'layerwise-bitmap-deflate-jbig-v1'


def _square(total):
    resolution = math.isqrt(total)
    if resolution * resolution != total:
        raise ValueError(f'a support mask covers a square grid; {total} cells do not')
    return resolution


def _deflate(data):
    packer = zlib.compressobj(9, zlib.DEFLATED, -15)
    return packer.compress(data) + packer.flush()


def encode_support(support):
    """One level's mask (flat CPU bool tensor of R^2 cells) as its smallest stored form; the record decodes back."""
    if not isinstance(support, torch.Tensor) or support.device.type != 'cpu' or support.dtype != torch.bool \
            or support.ndim != 1 or support.numel() < 1:
        raise ValueError('a support mask is a nonempty flat CPU bool tensor')
    bits = support.numpy()
    total, selected = bits.size, int(bits.sum())
    record = dict(num_cells=total, resolution=_square(total), selected_count=selected)
    if selected == 0 or selected == total:
        record['encoding'] = 'all' if selected else 'none'
        return record
    raw = np.packbits(bits, bitorder='little').tobytes()
    forms = [('bitmap', raw), ('bitmap_deflate', _deflate(raw))]
    encoding, data = min(forms, key=lambda form: len(form[1]))  # min keeps the first of equal lengths
    record.update(encoding=encoding, data=torch.from_numpy(np.frombuffer(data, dtype=np.uint8).copy()))
    if not torch.equal(decode_support(record), support):
        raise AssertionError('the stored mask does not decode to the support')
    return record


def _check_geometry(record):
    total, resolution, selected = record['num_cells'], record['resolution'], record['selected_count']
    for value in (total, resolution, selected):
        if type(value) is not int:
            raise ValueError('support geometry must be integers')
    if total < 1 or resolution < 1 or resolution * resolution != total or not 0 <= selected <= total:
        raise ValueError(f'inconsistent support geometry: {total} cells, R = {resolution}, {selected} selected')
    return total, selected


def decode_support(record):
    """The flat CPU bool mask of one stored level."""
    total, selected = _check_geometry(record)
    encoding = record['encoding']
    if encoding in ('all', 'none'):
        if selected != (total if encoding == 'all' else 0):
            raise ValueError(f"a constant '{encoding}' mask must select {'every' if encoding == 'all' else 'no'} cell")
        return torch.full((total,), encoding == 'all', dtype=torch.bool)
    if encoding == 'jbig1':
        raise RuntimeError('this checkpoint stores a JBIG1 mask; reading it needs the libjbig bridge, which is not '
                           'part of this build')
    if encoding not in ('bitmap', 'bitmap_deflate'):
        raise ValueError(f'unknown support encoding {encoding!r}')
    payload = record['data']
    if not isinstance(payload, torch.Tensor) or payload.dtype != torch.uint8 or payload.ndim != 1:
        raise ValueError('a stored mask is a flat uint8 tensor')
    data = payload.detach().cpu().numpy().tobytes()
    size = (total + 7) // 8
    if encoding == 'bitmap_deflate':
        inflater = zlib.decompressobj(-15)
        try:
            data = inflater.decompress(data, size + 1)
        except zlib.error as error:
            raise ValueError('the DEFLATE stream of a mask is corrupt') from error
        if not inflater.eof or inflater.unused_data or inflater.unconsumed_tail:
            raise ValueError('a DEFLATE mask stream must end exactly at its end')
    if len(data) != size:
        raise ValueError(f'a bitmap of {total} cells holds {size} bytes, not {len(data)}')
    if total % 8 and data[-1] >> (total % 8):
        raise ValueError('the padding bits of a bitmap must be zero')
    bits = np.unpackbits(np.frombuffer(data, dtype=np.uint8), bitorder='little', count=total)
    if int(bits.sum()) != selected:
        raise ValueError('the decoded mask selects a different number of cells than recorded')
    return torch.from_numpy(bits.astype(bool))


def encode_supports(supports):
    return [encode_support(support) for support in supports]


def decode_supports(artifact):
    """Every level's mask of a checkpoint (the layerwise records, or the older one-bitmap-per-level form)."""
    counts = artifact['support_num_cells']
    if 'support_encodings' in artifact:
        if artifact.get('support_storage_version') != STORAGE_VERSION:
            raise ValueError(f"support storage {artifact.get('support_storage_version')!r} is not {STORAGE_VERSION!r}")
        records = artifact['support_encodings']
        if len(records) != len(counts):
            raise ValueError('one support record per level is required')
        supports = [decode_support(record) for record in records]
    else:
        bitmaps = artifact['support_bitmaps']
        if len(bitmaps) != len(counts):
            raise ValueError('one support bitmap per level is required')
        supports = []
        for bits, count in zip(bitmaps, counts):
            if type(count) is not int or count < 1 or bits.dtype != torch.uint8 or bits.ndim != 1 \
                    or bits.numel() != (count + 7) // 8:
                raise ValueError('a legacy support bitmap does not match its cell count')
            unpacked = np.unpackbits(bits.detach().cpu().numpy(), bitorder='little', count=count)
            supports.append(torch.from_numpy(unpacked.astype(bool)))
    if [support.numel() for support in supports] != list(counts):
        raise ValueError('the masks do not have the recorded cell counts')
    config = artifact['configuration']
    if config['representation'] != 'hash_grid' and config.get('resolutions') is not None:
        if list(counts) != [r * r for r in config['resolutions']]:
            raise ValueError("the masks do not match the configuration's resolutions")
    return supports


def restore_support_record(artifact):
    """The support record (payload fields plus the decoded masks) of a checkpoint."""
    return dict(artifact['support_payload'], supports=decode_supports(artifact))


def fp16_parameters(model):
    """The model's parameters as fp16 CPU tensors, by name (the checkpoint's inference payload)."""
    return {name: p.detach().to('cpu', torch.float16).clone() for name, p in model.named_parameters()}


def export_checkpoint(path, model, config, settings, support_record, epoch, optimizer_steps, metrics, metadata=None):
    """Write the final fp16 checkpoint and verify it by reading it back: configuration, masks (and the rest of the
    support record) and every parameter's bytes must survive the round trip.  Returns the artifact written."""
    supports = support_record['supports']
    artifact = {'version': ARTIFACT_VERSION, 'configuration': config, 'settings': settings,
                'support_storage_version': STORAGE_VERSION, 'support_encodings': encode_supports(supports),
                'support_num_cells': [support.numel() for support in supports],
                'support_payload': {key: value for key, value in support_record.items() if key != 'supports'},
                'support_metadata': metadata if metadata is not None else support_record.get('metadata', {}),
                'parameters': fp16_parameters(model), 'checkpoint': 'latest', 'epoch': epoch,
                'optimizer_steps': optimizer_steps, 'metrics': metrics}
    path = Path(path)
    torch.save(artifact, path)
    back = torch.load(path, map_location='cpu', weights_only=True)
    if back['configuration'] != config:
        raise AssertionError('the configuration changed in the checkpoint round trip')
    restored = restore_support_record(back)
    if not all(torch.equal(a, b) for a, b in zip(restored['supports'], supports)) or \
            {k: v for k, v in restored.items() if k != 'supports'} != artifact['support_payload']:
        raise AssertionError('the support record changed in the checkpoint round trip')
    for name, value in artifact['parameters'].items():
        if not torch.equal(value.view(torch.uint16), back['parameters'][name].view(torch.uint16)):
            raise AssertionError(f'parameter {name} changed in the checkpoint round trip')
    return artifact


def load_parameters(model, artifact):
    """Copy a checkpoint's fp16 parameters into a model with the same parameter names."""
    saved = artifact['parameters']
    with torch.no_grad():
        own = dict(model.named_parameters())
        if set(own) != set(saved):
            raise ValueError(f'parameter names differ: model {sorted(own)}, checkpoint {sorted(saved)}')
        for name, parameter in own.items():
            parameter.copy_(saved[name].to(device=parameter.device, dtype=parameter.dtype))


def storage_statistics(records):
    """Per-level mask storage of a list of support records."""
    layers = [dict(level=i, resolution=r['resolution'], selected_count=r['selected_count'], encoding=r['encoding'],
                   bitmap_bytes=(r['num_cells'] + 7) // 8, payload_bytes=r['data'].numel() if 'data' in r else 0)
              for i, r in enumerate(records)]
    return dict(version=STORAGE_VERSION, selection_rule='smallest serialized stream; raw bitmap wins ties',
                layers=layers, bitmap_bytes=sum(x['bitmap_bytes'] for x in layers),
                payload_bytes=sum(x['payload_bytes'] for x in layers))
