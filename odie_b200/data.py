"""Targets, sampling and the seeded synthetic images of the benchmark configs.

ByteTarget and the batch samplers follow odie/data.py:9-80.  The reference
measures on DIV2K and gigapixel photographs that are not available here; the
synthetic generators below stand in for them with the shapes and value
distributions the benchmark configurations name (seeded, deterministic).
"""
import math

import torch


class ByteTarget:
    """RGB8 target [N, 3]; indexing returns fp32 / 255 (odie/data.py:9-28)."""

    def __init__(self, data):
        if data.dtype != torch.uint8 or data.ndim != 2 or data.shape[1] != 3:
            raise ValueError('Expected RGB8 Nx3 target')
        self.data, self.shape, self.device = data, data.shape, data.device

    def __getitem__(self, ids):
        return self.data[ids].float() / 255.

    def data_ptr(self):
        return self.data.data_ptr()

    def numel(self):
        return self.data.numel()

    def detach(self):
        return self

    def cpu(self):
        return self.data.cpu().float().div_(255.)


def stratified_batches(shape, batch, generator, device='cuda', steps=None):
    """One random pixel per square stratum per step (odie/data.py:63-80)."""
    height, width = shape
    side = int(batch ** .5)
    if batch < 1 or batch & (batch - 1) or side * side != batch:
        raise ValueError('Stratified sampling requires a square power-of-two batch size')
    slots = torch.arange(batch, device=device)
    strata = torch.stack((slots % side, slots // side), dim=1).float() / side
    scale = torch.tensor((width, height), dtype=torch.float32, device=device)
    count = (height * width + batch - 1) // batch if steps is None else steps
    for _ in range(count):
        uv = torch.rand((batch, 2), device=device, generator=generator) / side + strata
        xy = (uv * scale).long()
        yield xy[:, 1].clamp_(0, height - 1) * width + xy[:, 0].clamp_(0, width - 1)


def device_stratified_ids(shape, batch, seed, step, stream=None):
    """The stratified batch of (seed, step) drawn on the GPU (odie_stratified_ids): the strata of
    stratified_batches with a Philox4x32-10 stream instead of torch's generator; int64 CUDA tensor."""
    from . import _lib
    height, width = shape
    ids = torch.empty(batch, dtype=torch.int64, device='cuda')
    stream = stream if stream is not None else torch.cuda.current_stream()
    _lib.check(_lib.library().odie_stratified_ids(int(seed), int(step), width, height, batch, ids.data_ptr(),
                                                   stream.cuda_stream), 'odie_stratified_ids')
    return ids


def uniform_ids(shape, batch, generator, device='cuda'):
    """Uniform pixel ids in [0, H*W) (the benchmark configs' uniform coordinates)."""
    return torch.randint(0, shape[0] * shape[1], (batch,), device=device, generator=generator)


# ---------------------------------------------------------------- synthetic images
def _grid(height, width, device):
    y = torch.linspace(0, 1, height, device=device).view(-1, 1)
    x = torch.linspace(0, 1, width, device=device).view(1, -1)
    return x, y


def blobs_and_gratings(height, width, seed, blobs=64, gratings=8, device='cpu'):
    """Seeded sum of anisotropic Gaussian blobs and sinusoidal gratings, RGB in [0, 1] (float32 [H, W, 3])."""
    g = torch.Generator().manual_seed(seed)
    x, y = _grid(height, width, device)
    image = torch.zeros((height, width, 3), device=device)
    p = torch.rand((blobs, 9), generator=g)
    for b in range(blobs):
        cx, cy, sx, sy, th = p[b, 0], p[b, 1], .02 + .2 * p[b, 2], .02 + .2 * p[b, 3], math.pi * p[b, 4]
        c, s = torch.cos(th), torch.sin(th)
        dx, dy = x - cx, y - cy
        u, v = c * dx + s * dy, -s * dx + c * dy
        weight = torch.exp(-.5 * ((u / sx) ** 2 + (v / sy) ** 2))
        image += weight.unsqueeze(-1) * (p[b, 5:8].to(device) * 2 - 1)
    q = torch.rand((gratings, 6), generator=g)
    for k in range(gratings):
        freq, th, phase = 2 + 40 * q[k, 0], math.pi * q[k, 1], 2 * math.pi * q[k, 2]
        wave = torch.sin(2 * math.pi * freq * (torch.cos(th) * x + torch.sin(th) * y) + phase)
        image += .3 * wave.unsqueeze(-1) * q[k, 3:6].to(device)
    lo, hi = image.amin(), image.amax()
    return (image - lo) / (hi - lo)


def pink_noise(height, width, seed, device='cpu'):
    """1/f amplitude (1/f^2 power) noise, RGB, zero mean unit peak (float32 [H, W, 3])."""
    g = torch.Generator().manual_seed(seed)
    white = torch.randn((3, height, width), generator=g).to(device)
    spectrum = torch.fft.rfft2(white)
    fy = torch.fft.fftfreq(height, device=device).view(-1, 1)
    fx = torch.fft.rfftfreq(width, device=device).view(1, -1)
    f = torch.sqrt(fx * fx + fy * fy)
    f[0, 0] = 1.0
    noise = torch.fft.irfft2(spectrum / f, s=(height, width))
    noise = noise - noise.mean()
    return (noise / noise.abs().amax()).permute(1, 2, 0).contiguous()


def polygons(height, width, seed, count=200, device='cpu'):
    """Seeded random sharp-edged convex polygons with random colours (float32 [H, W, 3], [0, 1])."""
    g = torch.Generator().manual_seed(seed)
    x, y = _grid(height, width, device)
    image = torch.zeros((height, width, 3), device=device)
    for _ in range(count):
        sides = int(torch.randint(3, 8, (1,), generator=g))
        centre = torch.rand(2, generator=g)
        radius = .01 + .08 * float(torch.rand(1, generator=g))
        angles = torch.sort(torch.rand(sides, generator=g) * 2 * math.pi).values
        px = centre[0] + radius * torch.cos(angles)
        py = centre[1] + radius * torch.sin(angles)
        inside = torch.ones((height, width), dtype=torch.bool, device=device)
        for i in range(sides):
            x0, y0, x1, y1 = px[i], py[i], px[(i + 1) % sides], py[(i + 1) % sides]
            inside &= ((x1 - x0) * (y - y0) - (y1 - y0) * (x - x0)) >= 0
        colour = torch.rand(3, generator=g).to(device)
        image = torch.where(inside.unsqueeze(-1), colour, image)
    return image


def to_u8(image):
    return (image.clamp(0, 1) * 255).round().to(torch.uint8)


def synthetic_image(config, seed=1729, device='cpu'):
    """u8 [H*W, 3] target and (H, W) of a benchmark config name: c1, c2, c3."""
    if config == 'c1':
        h, w = 512, 512
        image = blobs_and_gratings(h, w, seed, device=device)
    elif config == 'c2':
        h, w = 1356, 2040
        base = blobs_and_gratings(h, w, seed, device=device)
        image = (.75 * base + .25 * (pink_noise(h, w, seed + 1, device=device) * .5 + .5)).clamp(0, 1)
    elif config == 'c3':
        h, w = 4096, 4096
        noise = pink_noise(h, w, seed, device=device) * .5 + .5
        shapes = polygons(h, w, seed + 2, device=device)
        mask = shapes.abs().sum(-1, keepdim=True) > 0
        image = torch.where(mask, shapes, noise).clamp(0, 1)
    elif isinstance(config, tuple):
        h, w = config
        image = blobs_and_gratings(h, w, seed, blobs=8, gratings=2, device=device)
    else:
        raise ValueError('unknown synthetic config ' + str(config))
    return to_u8(image).reshape(-1, 3), (h, w)


def procedural_image(shape, seed=1729, row0=0, rows=None, device='cuda'):
    """Rows [row0, row0 + rows) of the seeded procedural image of `shape` (odie_procedural_image: fractal
    1/f^2 noise, sharp-edged Voronoi regions, a 64 x 64-cell texture atlas) as a CUDA u8 [rows * W, 3]
    tensor.  The gigapixel benchmark's stand-in: every pixel depends only on (seed, column, row, shape), so
    each rank draws exactly its own band of one image."""
    from . import _lib
    height, width = shape
    rows = height - row0 if rows is None else rows
    out = torch.empty((rows * width, 3), dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream()
    _lib.check(_lib.library().odie_procedural_image(int(seed), width, height, row0, rows, out.data_ptr(),
                                                     stream.cuda_stream), 'odie_procedural_image')
    return out
