"""Single fp32 hash grid with an fp32 MLP, trained through the native library (odie_hashgrid32_*).

The hash-grid encoding of odie/hash_grid.py:8-80 (layout odie/config.py:83-94) in fp32: 16 levels of 2
features, tables initialised U(-1e-4, 1e-4); an MLP 32 -> 64 -> 64 -> 3 without biases (the TCNN
FullyFusedMLP topology, seeded Xavier-uniform weights) with ReLU hidden layers and a sigmoid output.
Training draws uniform coordinates in [0, 1)^2 on the device (or takes the caller's), samples the fp32
target image bilinearly, minimises the mean squared error and updates every parameter with Adam
(torch.optim.Adam's update, betas and eps from the configuration).

`HashGrid32` holds the parameters (fp32 CUDA tensors the library updates in place); `HashGrid32Trainer` owns
the library handle.  There is no CPU path: without the built library every call raises.
"""
import json
import math

import torch
from torch import nn

from . import _lib
from .layout import hash_levels

HEAD_SHAPES = [(64, 32), (64, 64), (3, 64)]
HEAD_PARAMS = sum(o * i for o, i in HEAD_SHAPES)  # 6336

C1_ENCODING = dict(otype='HashGrid', n_levels=16, n_features_per_level=2, log2_hashmap_size=19, base_resolution=16,
                   per_level_scale=1.5)


def c1_config(seed=1729, batch=1 << 18):
    """The single fp32 hash grid's configuration: T = 2^19, base 16, scale 1.5, Adam lr 1e-2, betas 0.9 / 0.99,
    eps 1e-15, 2^18 coordinates per step."""
    return dict(representation='hash_grid_fp32', hash_encoding=dict(C1_ENCODING), seed=seed, grid_init=1e-4,
                grid_lr=1e-2, head_lr=1e-2, beta1=0.9, beta2=0.99, eps=1e-15, batch_size=batch)


def xavier_heads(seed):
    """W1 [64][32] | W2 [64][64] | W3 [3][64], each U(-b, b) with b = sqrt(6 / (in + out)), from one seeded
    CPU generator."""
    generator = torch.Generator().manual_seed(int(seed))
    chunks = []
    for out_dim, in_dim in HEAD_SHAPES:
        bound = math.sqrt(6.0 / (in_dim + out_dim))
        chunks.append(((torch.rand((out_dim, in_dim), generator=generator) * 2 - 1) * bound).flatten())
    return torch.cat(chunks)


class HashGrid32(nn.Module):
    """Parameters and forward of the single fp32 hash grid (fp32 table `grid`, fp32 `heads`)."""

    def __init__(self, config, device='cuda'):
        super().__init__()
        self.config = dict(config)
        self.records, self.total = hash_levels(config['hash_encoding'])
        if len(self.records) != 16 or any(r['features'] != 2 for r in self.records):
            raise ValueError('the fp32 hash grid has 16 levels of 2 features')
        seed = int(config['seed'])
        init = float(config.get('grid_init', 1e-4))
        table = (torch.rand(self.total, generator=torch.Generator().manual_seed(seed)) * 2 - 1) * init
        self.grid = nn.Parameter(table.to(device))
        self.heads = nn.Parameter(xavier_heads((seed + 4000037) % 2 ** 31).to(device))
        self._runtime = None

    def matrices(self):
        out, offset = [], 0
        for out_dim, in_dim in HEAD_SHAPES:
            out.append(self.heads[offset:offset + out_dim * in_dim].view(out_dim, in_dim))
            offset += out_dim * in_dim
        return out

    @torch.no_grad()
    def forward(self, coordinates):
        """fp32 RGB [n, 3] at fp32 coordinates [n, 2] (odie_hashgrid32_decode)."""
        if self._runtime is None:
            raise RuntimeError('attach a HashGrid32Trainer first: the forward runs through its library handle')
        return self._runtime.decode(xy=coordinates)

    def storage_stats(self):
        return dict(actual_params=self.total + HEAD_PARAMS, grid_params=self.total, head_params=HEAD_PARAMS,
                    fp32_parameter_bytes=4 * (self.total + HEAD_PARAMS), adam_moment_bytes=8 * (self.total + HEAD_PARAMS),
                    plane_caps=[r['capacity'] for r in self.records], layout_version='hash-grid-fp32-v1',
                    addressing_version='instant-ngp-spatial-hash')


class HashGrid32Trainer:
    """The library's training handle of a HashGrid32 on an fp32 [H, W, 3] CUDA target image."""

    def __init__(self, model, image, capacity=None):
        if not (image.is_cuda and image.dtype == torch.float32 and image.dim() == 3 and image.shape[2] == 3):
            raise ValueError('the target is a CUDA fp32 [H, W, 3] image')
        self.model, self.image = model, image.contiguous()
        config = model.config
        self.capacity = int(capacity or config['batch_size'])
        settings = dict(image=self.image.data_ptr(), width=int(image.shape[1]), height=int(image.shape[0]),
                        grid=model.grid.data_ptr(), heads=model.heads.data_ptr(), total=int(model.total),
                        hash_encoding=config['hash_encoding'], capacity=self.capacity,
                        grid_lr=config['grid_lr'], head_lr=config['head_lr'], beta1=config['beta1'],
                        beta2=config['beta2'], eps=config['eps'])
        lib = _lib.library()
        self.handle = lib.odie_hashgrid32_create(json.dumps(settings).encode())
        if not self.handle:
            raise RuntimeError('odie_hashgrid32_create failed: ' + _lib.error())
        self.buffers = json.loads(lib.odie_hashgrid32_pointers(self.handle).decode())
        self.steps = 0
        model._runtime = self

    def step(self, step=None, xy=None, update=True, seed=None, stream=None):
        """One training step: `xy` CUDA fp32 [n, 2] coordinates, or None for the device's uniform draw of
        (seed, step) with the configured batch size.  Asynchronous; returns nothing."""
        step = self.steps if step is None else int(step)
        seed = int(self.model.config['seed']) if seed is None else int(seed)
        if xy is not None:
            if not (xy.is_cuda and xy.dtype == torch.float32 and xy.dim() == 2 and xy.shape[1] == 2):
                raise ValueError('coordinates are a CUDA fp32 [n, 2] tensor')
            xy = xy.contiguous()
        n = self.capacity if xy is None else xy.shape[0]
        _lib.check(_lib.library().odie_hashgrid32_step(self.handle, seed, step, n, _lib.ptr(xy), int(bool(update)),
                                                       _lib.stream_handle(stream)), 'odie_hashgrid32_step')
        self.steps = step + 1

    def update(self, stream=None):
        """Adam on the gradients accumulated by steps taken with update=False."""
        _lib.check(_lib.library().odie_hashgrid32_update(self.handle, _lib.stream_handle(stream)),
                   'odie_hashgrid32_update')

    def decode(self, xy=None, begin=0, n=None, out=None, stream=None):
        """fp32 RGB [n, 3] at coordinates xy, or at the pixel centres of pixels [begin, begin + n)."""
        if xy is not None:
            xy = xy.contiguous()
            n = xy.shape[0]
        elif n is None:
            n = self.image.shape[0] * self.image.shape[1] - begin
        out = torch.empty((n, 3), dtype=torch.float32, device=self.image.device) if out is None else out
        _lib.check(_lib.library().odie_hashgrid32_decode(self.handle, begin, n, _lib.ptr(xy), out.data_ptr(),
                                                         _lib.stream_handle(stream)), 'odie_hashgrid32_decode')
        return out

    def read(self, name, count, dtype=torch.float32, stream=None):
        """A copy of one library-owned device buffer (grid_grad, head_grad, squares, xy, dx, moments ...)."""
        out = torch.empty(count, dtype=dtype, device=self.image.device)
        _lib.check(_lib.library().odie_copy(out.data_ptr(), int(self.buffers[name]), out.numel() * out.element_size(),
                                            _lib.stream_handle(stream)), 'odie_copy')
        return out

    def loss(self, n=None, stream=None):
        """Mean squared error of the last step's n coordinates (a device scalar)."""
        return self.read('squares', n or self.capacity, stream=stream).mean()

    def close(self):
        if getattr(self, 'handle', None):
            torch.cuda.synchronize()
            _lib.library().odie_hashgrid32_destroy(self.handle)
            self.handle = None
        if self.model._runtime is self:
            self.model._runtime = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def c1_image(seed=1729, device='cuda'):
    """The single fp32 hash grid's target: the seeded 512 x 512 sum of 64 anisotropic Gaussian blobs and 8
    sinusoidal gratings scaled to [0, 1], fp32 [H, W, 3]."""
    from .data import blobs_and_gratings
    return blobs_and_gratings(512, 512, seed).to(device).contiguous()
