"""GPU parity of the device stratified sampler (odie_stratified_ids, odie_step_stratified) against its
restatement in the oracle, and of the fused input stage against the step on the same ids."""
import numpy as np
import pytest
import torch

from odie_b200 import _lib
from odie_b200.data import device_stratified_ids
from oracle import oracle
from tests.test_gpu_experts import SHAPE, setup

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize('shape,n,seed,step', [((1356, 2040), 1 << 20, 1729, 0), ((1356, 2040), 1 << 10, 7, 12345),
                                               ((4096, 4096), 1 << 16, 2 ** 40 + 3, 2 ** 33 + 1), ((5, 7), 4, 0, 1),
                                               ((2, 2), 1, 1, 1)])
def test_ids_match_oracle(cuda, shape, n, seed, step):
    ids = device_stratified_ids(shape, n, seed, step)
    torch.cuda.synchronize()
    want = oracle.stratified_ids(seed, step, shape[1], shape[0], n)
    assert np.array_equal(ids.cpu().numpy(), want)


def test_ids_stay_in_their_strata_and_vary_by_step(cuda):
    shape, n = (1356, 2040), 1 << 16
    side = 256
    a = device_stratified_ids(shape, n, 11, 3).cpu().numpy()
    b = device_stratified_ids(shape, n, 11, 3).cpu().numpy()
    c = device_stratified_ids(shape, n, 11, 4).cpu().numpy()
    assert np.array_equal(a, b), 'the same (seed, step) must give the same batch'
    # independent draws land on the same pixel with probability ~ strata / pixels (1 / pixels per stratum)
    assert (a != c).mean() > 1 - 2 * n / (shape[0] * shape[1]), 'another step must give another batch'
    j = np.arange(n)
    x, y = a % shape[1], a // shape[1]
    sx, sy = j % side, j // side
    # pixel within its stratum's span (one pixel of slack for the fp32 rounding of uv, as in the reference)
    assert np.all(x >= np.floor(sx * shape[1] / side) - 1) and np.all(x <= np.ceil((sx + 1) * shape[1] / side))
    assert np.all(y >= np.floor(sy * shape[0] / side) - 1) and np.all(y <= np.ceil((sy + 1) * shape[0] / side))


def test_ids_reject_non_square_batches(cuda):
    for n in (3, 8, 1 << 11):
        with pytest.raises(RuntimeError):
            device_stratified_ids((64, 64), n, 1, 1)


@pytest.mark.parametrize('model_kind', ['experts', 'planes'])
def test_fused_step_input_matches_step_on_the_same_ids(cuda, model_kind):
    if model_kind == 'experts':
        config, model, rgb, opt = setup(experts=4, batch=1024)
        shape = SHAPE
    else:
        from tests import test_gpu_step
        config, model, rgb, opt = test_gpu_step.setup(batch=1024)[:4]
        shape = test_gpu_step.SHAPE
    n = 1024
    ids = device_stratified_ids(shape, n, 99, 5)
    opt.check(opt.lib.odie_step(opt.handle, ids.data_ptr(), n, 0))  # update 0: weights stay as they are
    torch.cuda.synchronize()
    plain = [opt.copied(name, shape, torch.float32).cpu().numpy() for name, shape in
             (('xy', (n, 2)), ('target', (n, 3)), ('squares', (n,)))]
    opt.check(opt.lib.odie_step_stratified(opt.handle, 99, 5, n, 0))
    torch.cuda.synchronize()
    fused = [opt.copied(name, shape, torch.float32).cpu().numpy() for name, shape in
             (('xy', (n, 2)), ('target', (n, 3)), ('squares', (n,)))]
    for name, p, f in zip(('coordinates', 'targets', 'squares'), plain, fused):
        assert np.array_equal(p.view(np.uint32), f.view(np.uint32)), f'{name} differ'
    with pytest.raises(RuntimeError):
        opt.step_stratified(99, 5, 1000)  # not a square power of two
    opt.close()
    assert _lib.library() is not None
