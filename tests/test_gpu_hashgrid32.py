"""The single fp32 hash grid on the GPU (odie_hashgrid32_*) against the oracle, on the benchmark configuration
itself: T = 2^19, 16 levels, the seeded 512 x 512 image, Philox uniform coordinates.

Criteria: coordinates bit-exact; predictions (features, two ReLU layers, logits: fma chains in the oracle's
order, then CUDA's expf) within 1e-6 relative; per-coordinate losses and feature gradients within 1e-5
relative with a 1e-5 x rms floor (the sigmoid's last-ulp differences pass through y - target); weight and
grid gradients within 1e-5 of the sum of their terms' magnitudes plus that floor carried through the sums;
Adam bit-exact given the step's gradients."""
import numpy as np
import pytest
import torch

from cases import close, close_bound
from odie_b200.hashgrid32 import HashGrid32, HashGrid32Trainer, c1_config, c1_image
from oracle import oracle

pytestmark = pytest.mark.gpu

SEED = 1729


def make(capacity, grid_scale=0.3, seed=SEED):
    """The configuration's model with a wider table initialisation (so the features reach every hidden unit's
    nonlinearity) and its trainer."""
    model = HashGrid32(c1_config(seed=seed, batch=capacity))
    with torch.no_grad():
        g = torch.Generator(device='cuda').manual_seed(seed)
        model.grid.uniform_(-grid_scale, grid_scale, generator=g)
    image = c1_image(seed)
    return model, image, HashGrid32Trainer(model, image, capacity)


def gradient_bounds(r, xy, records, total, rtol=1e-5, floor=1e-5):
    """Per-entry bounds of the head and grid gradients (see the module docstring)."""
    d = {k: np.abs(r[k].astype(np.float64)) for k in ('dz', 'dh2', 'dh1', 'dx', 'h1', 'h2', 'features')}
    rms = {k: float(np.sqrt(np.mean(r[k].astype(np.float64) ** 2))) for k in ('dz', 'dh2', 'dh1', 'dx')}
    sums = np.concatenate([(floor * rms['dh1']) * np.tile(d['features'].sum(0), (64, 1)).reshape(-1),
                           (floor * rms['dh2']) * np.tile(d['h1'].sum(0), (64, 1)).reshape(-1),
                           (floor * rms['dz']) * np.tile(d['h2'].sum(0), (3, 1)).reshape(-1)])
    head = 2 * rtol * r['head_magnitude'] + sums
    weights = oracle.hg32_scatter(xy, np.ones((xy.shape[0], 32)), records, total)
    grid = 2 * rtol * r['grid_magnitude'] + floor * rms['dx'] * weights
    return head, grid


@pytest.mark.parametrize('n', [4096, 1000])
def test_step_matches_oracle(cuda, n):
    model, image, trainer = make(n)
    grid0, heads0 = model.grid.detach().cpu().numpy(), model.heads.detach().cpu().numpy()
    trainer.step(step=3, update=False)
    torch.cuda.synchronize()
    xy = trainer.read('xy', 2 * n).view(n, 2).cpu().numpy()
    assert np.array_equal(xy, oracle.uniform_xy(SEED, 3, n)), 'uniform coordinates differ from Philox'
    r = oracle.hg32_step(image.cpu().numpy(), xy, grid0, heads0, model.records)
    close(trainer.read('squares', n).cpu().numpy(), r['squares'], 1e-5, 1e-5, 'per-coordinate loss')
    close(trainer.read('dx', 32 * n).view(n, 32).cpu().numpy(), r['dx'], 1e-5, 1e-5, 'feature gradients')
    head_bound, grid_bound = gradient_bounds(r, xy, model.records, model.total)
    close_bound(trainer.read('head_grad', 6336).cpu().numpy(), r['head_grad'], head_bound, 'head gradient')
    close_bound(trainer.read('grid_grad', model.total).cpu().numpy(), r['grid_grad'], grid_bound, 'grid gradient')
    # the prediction at the step's coordinates
    y = trainer.decode(xy=torch.from_numpy(xy).cuda()).cpu().numpy()
    close(y, r['y'], 1e-6, 0.0, 'prediction')
    trainer.close()


def test_decode_pixels_matches_oracle(cuda):
    model, image, trainer = make(1024)
    h, w = image.shape[:2]
    begin, n = 511 * w - 100, 300  # the end of one row and the start of the next
    rgb = trainer.decode(begin=begin, n=n).cpu().numpy()
    ids = np.arange(begin, begin + n)
    xy = oracle.coords(ids, w, h)
    r = oracle.hg32_step(image.cpu().numpy(), xy, model.grid.detach().cpu().numpy(),
                         model.heads.detach().cpu().numpy(), model.records)
    close(rgb, r['y'], 1e-6, 0.0, 'decoded pixels')
    with pytest.raises(RuntimeError):
        trainer.decode(begin=h * w - 10, n=20)  # past the image
    trainer.close()


def test_adam_matches_oracle_given_gradients(cuda):
    """Dense Adam (betas 0.9 / 0.99, eps 1e-15, lr 1e-2) on the step's own gradients, twice: bit-exact."""
    model, image, trainer = make(2048)
    p, q = model.grid.detach().cpu().numpy(), model.heads.detach().cpu().numpy()
    state = [(p, np.zeros_like(p), np.zeros_like(p), np.zeros(p.size, np.uint32)),
             (q, np.zeros_like(q), np.zeros_like(q), np.zeros(q.size, np.uint32))]
    for step in range(2):
        trainer.step(step=step, update=False)
        g = [trainer.read('grid_grad', model.total).cpu().numpy(), trainer.read('head_grad', 6336).cpu().numpy()]
        trainer.update()
        torch.cuda.synchronize()
        for k, (param, grad) in enumerate(zip((model.grid, model.heads), g)):
            pk, mk, vk, sk = state[k]
            pk, mk, vk, sk, _ = oracle.adam(pk, mk, vk, sk, grad, 1.0, 1e-2, False, beta1=0.9, beta2=0.99, eps=1e-15)
            state[k] = (pk, mk, vk, sk)
            assert np.array_equal(param.detach().cpu().numpy().view(np.uint32), pk.view(np.uint32)), \
                f'Adam step {step} of {"grid" if k == 0 else "heads"} differs'
        assert not trainer.read('grid_grad', model.total).any(), 'the update consumes the gradient'
    trainer.close()


def test_full_batch_matches_oracle(cuda):
    """The benchmark's own step: 2^18 coordinates on the configuration's initialisation (tables U(-1e-4, 1e-4))."""
    n = 1 << 18
    model = HashGrid32(c1_config(seed=SEED, batch=n))
    image = c1_image(SEED)
    trainer = HashGrid32Trainer(model, image, n)
    grid0, heads0 = model.grid.detach().cpu().numpy(), model.heads.detach().cpu().numpy()
    trainer.step(step=0, update=False)
    torch.cuda.synchronize()
    xy = trainer.read('xy', 2 * n).view(n, 2).cpu().numpy()
    assert np.array_equal(xy, oracle.uniform_xy(SEED, 0, n))
    r = oracle.hg32_step(image.cpu().numpy(), xy, grid0, heads0, model.records)
    close(trainer.read('squares', n).cpu().numpy(), r['squares'], 1e-5, 1e-5, 'per-coordinate loss')
    close(trainer.read('dx', 32 * n).view(n, 32).cpu().numpy(), r['dx'], 1e-5, 1e-5, 'feature gradients')
    head_bound, grid_bound = gradient_bounds(r, xy, model.records, model.total)
    close_bound(trainer.read('head_grad', 6336).cpu().numpy(), r['head_grad'], head_bound, 'head gradient')
    close_bound(trainer.read('grid_grad', model.total).cpu().numpy(), r['grid_grad'], grid_bound, 'grid gradient')
    trainer.close()


def test_training_reduces_the_loss(cuda):
    n = 1 << 16
    model = HashGrid32(c1_config(seed=SEED, batch=n))
    trainer = HashGrid32Trainer(model, c1_image(SEED), n)
    losses = []
    for step in range(60):
        trainer.step(step=step)
        if step in (0, 59):
            losses.append(float(trainer.loss()))
    assert losses[1] < 0.25 * losses[0], losses
    assert int(trainer.read('error_flag', 1, dtype=torch.int32)) == 0
    trainer.close()
