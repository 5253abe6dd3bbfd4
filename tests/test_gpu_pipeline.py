"""Pipeline mode of the routed-expert runtime (odie_create's "pipeline": 1): each step's backward branches run on
the runtime's own streams while the next step's forward starts.  The same steps on two identically seeded
c2-experts models, one pipelined and one not, must train the same model: the step losses within 1e-5 relative, and
every parameter within 1e-5 absolute.  Both runs sum their gradients in an order the hardware picks (scatter
atomics; the heads' weight gradients accumulated by three warpgroups), and Adam turns a gradient whose terms nearly
cancel into an update of either sign, so up to 1 % of the entries (at least 8) may differ by more, each by at most
the updates' own size (2 x steps x lr); stale parameters read by a step would move the losses instead.  The
pipelined runtime must also leave nothing running once joined: its parameters stay put across a further wait."""
import numpy as np
import pytest
import torch

from odie_b200 import workloads
from odie_b200.data import ByteTarget, stratified_batches
from odie_b200.model import RoutedExperts
from odie_b200.native_backend import NativeOptimizer

pytestmark = pytest.mark.gpu
N = 1 << 14
STEPS = 4


def train(pipeline, ids):
    config, rgb, shape = workloads.c2_experts(batch=N)
    model = RoutedExperts(config)
    opt = NativeOptimizer(model, ByteTarget(rgb.cuda()), shape, config, [model.grid], batch=N, pipeline=pipeline)
    losses = [opt.train_batch(batch) for batch in ids]
    opt.join()
    torch.cuda.synchronize()
    params = [t.detach().clone() for t in (model.grid, model.router_grid, model.gate.params, model.decoder.params)]
    assert opt.copied('error_flag', (1,), torch.int32).item() == 0
    return opt, model, torch.stack(losses).cpu().numpy(), params


def test_pipelined_steps_train_the_same_model(cuda):
    config, _, shape = workloads.c2_experts(batch=N)
    ids = list(stratified_batches(shape, N, torch.Generator(device='cuda').manual_seed(21), steps=STEPS))
    opt_a, _, loss_a, params_a = train(False, ids)
    opt_b, model_b, loss_b, params_b = train(True, ids)
    assert np.allclose(loss_a, loss_b, rtol=1e-5, atol=0), (loss_a, loss_b)
    rates = (config['grid_lr'], config['grid_lr'], config['gate_lr'], config['decoder_lr'])
    for name, a, b, lr in zip(('grid', 'router grid', 'router MLP', 'decoder'), params_a, params_b, rates):
        diff = (a - b).abs()
        far = int((diff > 1e-5).sum())
        worst = float(diff.max())
        assert far <= max(8, a.numel() // 100), f'{name}: {far} of {a.numel()} entries differ by more than 1e-5'
        assert worst <= 2 * STEPS * lr * 1.001, f'{name}: an entry differs by {worst}'
    # joined: nothing of the pipelined steps is still running
    torch.cuda.synchronize()
    assert torch.equal(model_b.grid.detach(), params_b[0]) and torch.equal(model_b.router_grid.detach(), params_b[1])
    opt_a.close()
    opt_b.close()


def test_pipeline_needs_library_owned_gradients(cuda):
    config, rgb, shape = workloads.c2_experts(batch=N)
    model = RoutedExperts(config)
    head_grad = torch.zeros(model.gate.params.numel() + model.decoder.params.numel(), device='cuda')
    with pytest.raises(RuntimeError, match='pipeline mode'):
        NativeOptimizer(model, ByteTarget(rgb.cuda()), shape, config, [model.grid], batch=N, head_grad=head_grad,
                        pipeline=True)
