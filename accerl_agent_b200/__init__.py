"""accerl_agent_b200: a Blackwell (sm_100a) native asynchronous online-RL framework for LLM agents.

Layout
------
core/      RLSample data contract, CLI flags and validation, metrics sinks
algo/      varlen packing, policy objectives (PPO/GIPO/SAPO + k3 KL), advantages, LR schedule
replay/    sharded replay buffer and rollout statistics
env/       seeded synthetic text-game environment and the TextWorld adapter
rollout/   interruptible (abort/resubmit, versioned) generation, paged-KV engine, rollout workers
runtime/   process actors (Ray-free), launcher, rendezvous helpers
models/    Qwen2 dense / Qwen2-MoE / Qwen3-MoE decoder built on the native ops, HF safetensors I/O
ops/       Python bindings of the sm_100a CUDA kernels (csrc/) plus fp32 PyTorch oracles
parallel/  FSDP-style flat-shard runtime, symmetric peer memory, weight sync, expert parallel
trainer/   the RL train worker (varlen + padded optimizer steps, checkpointing)
utils/     timing (CUDA events, max over ranks), clocks sampling, seeding
"""

__version__ = "0.1.0"
