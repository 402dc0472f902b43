"""Distribution: process groups, tensor-parallel collectives (NCCL baseline and fused P2P)."""
