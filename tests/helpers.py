"""Helpers shared by the GPU parity tests."""
import torch


def bf16_ulps(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """Distance between two bf16 tensors in units of the last place (sign-magnitude order)."""
    ia = a.contiguous().view(torch.int16).to(torch.int32)
    ib = b.contiguous().view(torch.int16).to(torch.int32)
    ia = torch.where(ia < 0, -(ia & 0x7FFF), ia)
    ib = torch.where(ib < 0, -(ib & 0x7FFF), ib)
    return (ia - ib).abs()


def load_oracle_state(dec, oracle):
    """Copy the oracle's caches into a Decoder (layouts of the reference kernels)."""
    n = oracle.position
    dec.reset()
    dec._dn_states.copy_(oracle.dn_states_ref_layout())
    dec._conv_bufs.copy_(oracle.conv_ref_layout())
    dec._fa_k_cache[:, :, :n].copy_(torch.stack(oracle.k_cache))
    dec._fa_v_cache[:, :, :n].copy_(torch.stack(oracle.v_cache))
    dec._position = n
