"""MSE / PSNR / SSIM with the reference's signatures (manbo/metric.py), on B200 kernels."""
from repo_b200.metric import mse_loss as mse_loss_tilelang
from repo_b200.metric import psnr, ssim

__all__ = ["mse_loss_tilelang", "psnr", "ssim"]
