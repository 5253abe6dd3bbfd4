"""Full-image evaluation and decode (odie/evaluation.py, scripts/reconstruct.py)."""
import math

import torch


def coordinates(shape, ids):
    """Endpoint coordinates x = (id mod W)/(W-1), y = floor(id/W)/(H-1) (odie/evaluation.py:6-9)."""
    height, width = shape
    return torch.stack((ids.remainder(width).float() / (width - 1),
                        torch.div(ids, width, rounding_mode='floor').float() / (height - 1)), dim=1)


@torch.no_grad()
def evaluate(model, target, shape, batch_size, return_image=False):
    """Batched full-image MSE/PSNR through the module path (odie/evaluation.py:12-36)."""
    was_training = model.training
    model.eval()
    data = getattr(target, 'data', target)
    pixels = data.shape[0]
    total = torch.zeros((), dtype=torch.float64, device=data.device)
    image = torch.empty((pixels, 3), dtype=torch.float32) if return_image else None
    for begin in range(0, pixels, batch_size):
        ids = torch.arange(begin, min(begin + batch_size, pixels), device=data.device)
        prediction = model(coordinates(shape, ids)).float()
        total += (prediction - target[ids]).square().double().sum()
        if image is not None:
            image[begin:begin + ids.numel()] = prediction.cpu()
    mse = float(total.item() / (pixels * 3))
    if not math.isfinite(mse):
        raise FloatingPointError('Full-image RGB evaluation is nonfinite')
    model.train(was_training)
    return {'mse': mse, 'psnr_db': -10 * math.log10(mse) if mse else None}, image


@torch.no_grad()
def decode_image(optimizer, shape, chunk=1 << 24, rgb8=True):
    """Fused decode of the whole image through the native runtime into a device tensor [H*W, 3]."""
    pixels = shape[0] * shape[1]
    out = torch.empty((pixels, 3), dtype=torch.uint8 if rgb8 else torch.float32, device='cuda')
    for begin in range(0, pixels, chunk):
        count = min(chunk, pixels - begin)
        view = out[begin:begin + count]
        optimizer.decode(begin, count, rgb8=view if rgb8 else None, rgb=None if rgb8 else view)
    return out
