"""Rank layout of the pipeline trainer's roles and the GPU each local rank drives (reference train_pp.py:55-56,
1142-1204).

Ranks, in this order: learners (the pipeline-parallel x data-parallel training ranks), rollout actors, teachers,
LM servers, VAE servers. GPU numbers are the ones ``nvidia-smi`` prints: ``CUDA_DEVICE_ORDER=PCI_BUS_ID`` must be in
the environment before CUDA is initialised (``use_pci_bus_order`` sets it), otherwise CUDA numbers GPUs fastest
first. Placement rules, applied to the usable GPUs (all but ``skip_gpus``) with one local rank per usable GPU:

* the LM server (``lm_gpu``) and the VAE server (``vae_gpu``) get the GPUs named for them; the training ranks take
  the other usable GPUs in increasing order, the named servers come last;
* explicit actor GPUs (``actor_gpus``) are placed right after the learners;
* an explicit teacher GPU comes after the actors, before the LM / VAE servers;
* without any of these, local rank i drives usable GPU i.
"""
import os


def use_pci_bus_order():
    """Number GPUs as nvidia-smi does; call before anything initialises CUDA."""
    os.environ.setdefault("CUDA_DEVICE_ORDER", "PCI_BUS_ID")


class RankLayout:
    def __init__(self, world_all, actors=0, teachers=0, lm_servers=0, vae_servers=0, teacher_on_lm=False):
        self.world_all = world_all
        n = world_all - actors - teachers - lm_servers - vae_servers
        if n <= 0:
            raise ValueError("at least one learner rank is needed")
        self.learners = list(range(n))
        self.actors = list(range(n, n + actors))
        t0 = n + actors
        self.teachers = list(range(t0, t0 + teachers))
        self.lm_servers = list(range(t0 + teachers, world_all - vae_servers))
        self.vae_servers = list(range(world_all - vae_servers, world_all))
        if teacher_on_lm:
            self.teachers += self.lm_servers

    @property
    def n_learners(self):
        return len(self.learners)

    def role(self, rank):
        for name, ranks in (("learner", self.learners), ("actor", self.actors), ("lm", self.lm_servers),
                            ("vae", self.vae_servers), ("teacher", self.teachers)):
            if rank in ranks:
                return name
        raise ValueError(f"rank {rank} outside the layout of {self.world_all}")

    def lm_server_of(self, learner_rank):
        """LM server of a learner (round robin over the LM servers)."""
        return self.lm_servers[learner_rank % len(self.lm_servers)] if self.lm_servers else None

    def lm_clients(self, server, pp=1):
        """Learners served by an LM server: stage 0 of every pipeline (the stage that consumes LM states)."""
        return [r for r in self.learners if r % pp == 0 and self.lm_server_of(r // pp) == server]


def local_device(local_rank, n_dev, layout, skip_gpus=(), lm_gpu=-1, vae_gpu=-1, actor_gpus=(), teacher_gpu=-1):
    """GPU index (nvidia-smi numbering) for this local rank under the rules of the module docstring."""
    usable = [d for d in range(max(1, n_dev)) if d not in set(skip_gpus)]
    world_all = layout.world_all
    if skip_gpus and len(usable) != world_all:
        raise ValueError(f"--skip-gpus {list(skip_gpus)} leaves {len(usable)} GPUs for {world_all} ranks")
    tail = ([lm_gpu] if layout.lm_servers and lm_gpu >= 0 else []) + \
           ([vae_gpu] if layout.vae_servers and vae_gpu >= 0 else [])
    if len(set(tail)) != len(tail):
        raise ValueError("--lm-gpu and --vae-gpu must differ")
    one_each = len(usable) == world_all
    order = None
    if tail and one_each and all(d in usable for d in tail):
        order = [d for d in usable if d not in tail] + tail
    elif skip_gpus:
        order = list(usable)
    actor_gpus = list(actor_gpus)
    if actor_gpus:
        if not one_each:
            raise ValueError("explicit actor GPUs need one local GPU per rank")
        if len(set(actor_gpus)) != len(actor_gpus) or any(d not in usable or d in tail for d in actor_gpus):
            raise ValueError("actor GPUs must be distinct, usable and differ from the LM / VAE GPUs")
        order = [d for d in usable if d not in tail and d not in actor_gpus] + tail
        n = layout.n_learners
        order[n:n] = actor_gpus
    if teacher_gpu >= 0:
        if not one_each or teacher_gpu not in usable or teacher_gpu in tail + actor_gpus:
            raise ValueError("--teacher-gpu must be a usable GPU other than the LM / VAE / actor GPUs")
        if len(layout.teachers) != 1:
            raise ValueError("--teacher-gpu needs exactly one dedicated teacher rank")
        if layout.lm_servers and lm_gpu < 0:
            raise ValueError("--teacher-gpu needs an explicit --lm-gpu")
        if layout.actors and len(actor_gpus) != len(layout.actors):
            raise ValueError("explicit teacher placement needs explicit actor GPUs")
        order = [d for d in usable if d not in tail + actor_gpus + [teacher_gpu]] + actor_gpus + [teacher_gpu] + tail
    if order is None:
        return usable[local_rank % len(usable)]
    return order[local_rank]
