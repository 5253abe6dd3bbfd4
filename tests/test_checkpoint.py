"""The fp16 checkpoint format (odie_b200.checkpoint): mask storage pinned byte for byte to the reference's own
encoder (tests/golden/support_codec.npz, made by odie/support_codec.py), decoding and its refusals, and the full
export/reload round trip of a model."""
import numpy as np
import pytest
import torch

from odie_b200 import checkpoint

KEYS = ('r1_one', 'r8_all', 'r9_none', 'r37_random', 'r64_sparse', 'r5_single', 'r3_pad', 'r100_blocky')


@pytest.mark.parametrize('key', KEYS)
def test_mask_encoding_matches_reference(golden, key):
    g = golden('support_codec.npz')
    mask = torch.from_numpy(g[f'{key}_mask'].astype(bool))
    record = checkpoint.encode_support(mask)
    assert record['encoding'] == bytes(g[f'{key}_encoding']).decode()
    assert [record['num_cells'], record['resolution'], record['selected_count']] == g[f'{key}_meta'].tolist()
    data = record['data'].numpy() if 'data' in record else np.zeros(0, np.uint8)
    assert np.array_equal(data, g[f'{key}_data']), 'stored mask bytes differ from the reference encoder'
    assert torch.equal(checkpoint.decode_support(record), mask)


def test_both_stored_forms_occur(golden):
    g = golden('support_codec.npz')
    encodings = {bytes(g[f'{k}_encoding']).decode() for k in KEYS}
    assert {'all', 'none', 'bitmap', 'bitmap_deflate'} <= encodings


def test_decode_refuses_damaged_records():
    mask = torch.zeros(81, dtype=torch.bool)
    mask[::7] = True
    record = checkpoint.encode_support(mask)
    assert record['encoding'] == 'bitmap'
    bad_padding = dict(record, data=record['data'].clone())
    bad_padding['data'][-1] |= 0x80  # a bit past cell 80
    with pytest.raises(ValueError, match='padding'):
        checkpoint.decode_support(bad_padding)
    with pytest.raises(ValueError, match='different number'):
        checkpoint.decode_support(dict(record, selected_count=record['selected_count'] + 1))
    with pytest.raises(ValueError, match='square'):
        checkpoint.encode_support(torch.ones(10, dtype=torch.bool))
    with pytest.raises(RuntimeError, match='JBIG'):
        checkpoint.decode_support(dict(record, encoding='jbig1'))
    deflated = checkpoint.encode_support(torch.zeros(10000, dtype=torch.bool).index_fill_(0, torch.arange(5), True))
    assert deflated['encoding'] == 'bitmap_deflate'
    with pytest.raises(ValueError, match='end exactly'):
        checkpoint.decode_support(dict(deflated, data=torch.cat((deflated['data'], torch.zeros(3, dtype=torch.uint8)))))


def test_legacy_bitmaps_are_read():
    masks = [torch.ones(16, dtype=torch.bool), torch.tensor([1, 0, 0, 1, 1, 0, 0, 0, 1], dtype=torch.bool)]
    artifact = {'support_num_cells': [16, 9], 'configuration': {'representation': 'xy_planes', 'resolutions': [4, 3]},
                'support_bitmaps': [torch.from_numpy(np.packbits(m.numpy(), bitorder='little')) for m in masks]}
    decoded = checkpoint.decode_supports(artifact)
    assert all(torch.equal(a, b) for a, b in zip(decoded, masks))


class Tiny(torch.nn.Module):
    """Parameters named like the planes model's: grid, gate.params, decoder.params."""

    def __init__(self):
        super().__init__()
        self.grid = torch.nn.Parameter(torch.randn(1000) * 1e-3)
        self.gate = torch.nn.Module()
        self.gate.params = torch.nn.Parameter(torch.randn(32 * 32 + 16 * 32))
        self.decoder = torch.nn.Module()
        self.decoder.params = torch.nn.Parameter(torch.randn(32 * 64 + 64 * 64 + 16 * 64))


def test_export_round_trip(tmp_path):
    torch.manual_seed(0)
    model = Tiny()
    supports = [torch.ones(16, dtype=torch.bool), torch.rand(400) < .1, torch.zeros(900, dtype=torch.bool)]
    record = dict(supports=supports, plane_dims=[2, 2, 2], plane_node_caps=[16, 128, 8], metadata={'stage': 3})
    config = {'representation': 'xy_planes', 'resolutions': [4, 20, 30], 'n_levels': 3, 'seed': 1729}
    artifact = checkpoint.export_checkpoint(tmp_path / 'model_latest_fp16.pt', model, config, {'lr': 1e-2}, record,
                                            epoch=50, optimizer_steps=1234, metrics={'mse': 1e-3})
    back = torch.load(tmp_path / 'model_latest_fp16.pt', map_location='cpu', weights_only=True)
    assert set(back) == {'version', 'configuration', 'settings', 'support_storage_version', 'support_encodings',
                         'support_num_cells', 'support_payload', 'support_metadata', 'parameters', 'checkpoint',
                         'epoch', 'optimizer_steps', 'metrics'}
    assert back['version'] == 'packed-capacity-control-v1' and back['checkpoint'] == 'latest'
    assert back['support_storage_version'] == 'layerwise-bitmap-deflate-jbig-v1'
    assert back['support_num_cells'] == [16, 400, 900] and back['support_metadata'] == {'stage': 3}
    assert {r['encoding'] for r in back['support_encodings']} >= {'all', 'none'}
    assert set(back['parameters']) == {'grid', 'gate.params', 'decoder.params'}
    assert all(v.dtype == torch.float16 for v in back['parameters'].values())
    restored = checkpoint.restore_support_record(back)
    assert restored['plane_node_caps'] == [16, 128, 8] and torch.equal(restored['supports'][1], supports[1])
    fresh = Tiny()
    checkpoint.load_parameters(fresh, back)
    assert torch.equal(fresh.grid.detach(), model.grid.detach().half().float())
    stats = checkpoint.storage_statistics(artifact['support_encodings'])
    assert stats['bitmap_bytes'] == 2 + 50 + 113
