"""Flow-match scheduler of the denoise loop (投机采样/wam-p0-worktree/wan_va/
utils/scheduler.py:6-89, inference part). The schedule (sigmas, timesteps)
is host-side scalar setup, as in the reference; the step itself,
prev = sample + v * (sigma_next - sigma), runs on the device
(wamb_flow_step), in place.
"""
import torch

from . import _lib


class FlowMatchScheduler:
    def __init__(self, num_inference_steps=100, num_train_timesteps=1000, shift=3.0, sigma_max=1.0,
                 sigma_min=0.003 / 1.002, inverse_timesteps=False, extra_one_step=False,
                 reverse_sigmas=False):
        self.num_train_timesteps = num_train_timesteps
        self.shift, self.sigma_max, self.sigma_min = shift, sigma_max, sigma_min
        self.inverse_timesteps, self.extra_one_step = inverse_timesteps, extra_one_step
        self.reverse_sigmas = reverse_sigmas
        self.set_timesteps(num_inference_steps)

    def set_timesteps(self, num_inference_steps=100, denoising_strength=1.0, shift=None):
        """scheduler.py:33-62 without the exponential-shift / terminal options."""
        if shift is not None:
            self.shift = shift
        start = self.sigma_min + (self.sigma_max - self.sigma_min) * denoising_strength
        n = num_inference_steps + 1 if self.extra_one_step else num_inference_steps
        sig = torch.linspace(start, self.sigma_min, n)
        if self.extra_one_step:
            sig = sig[:-1]
        if self.inverse_timesteps:
            sig = torch.flip(sig, dims=[0])
        sig = self.shift * sig / (1 + (self.shift - 1) * sig)
        if self.reverse_sigmas:
            sig = 1 - sig
        self.sigmas = sig
        self.timesteps = sig * self.num_train_timesteps

    def delta(self, timestep, to_final=False):
        """sigma_next - sigma for `timestep` (scheduler.py:78-88)."""
        i = int(torch.argmin((self.timesteps - float(timestep)).abs()))
        sigma = float(self.sigmas[i])
        if to_final or i + 1 >= len(self.timesteps):
            nxt = 1.0 if (self.inverse_timesteps or self.reverse_sigmas) else 0.0
        else:
            nxt = float(self.sigmas[i + 1])
        return nxt - sigma

    def step_(self, model_output, timestep, sample, to_final=False):
        """In place: sample += model_output * (sigma_next - sigma); returns sample."""
        if sample.shape != model_output.shape or not (sample.is_contiguous() and model_output.is_contiguous()):
            raise ValueError("sample and model_output must be contiguous tensors of one shape")
        _lib.check(_lib.load().wamb_flow_step(
            sample.data_ptr(), int(sample.dtype == torch.float32), model_output.data_ptr(),
            int(model_output.dtype == torch.float32), sample.numel(), self.delta(timestep, to_final),
            _lib.stream_ptr()))
        return sample

    def step(self, model_output, timestep, sample, to_final=False):
        """Out of place, as the reference's step()."""
        return self.step_(model_output, timestep, sample.clone(), to_final)
