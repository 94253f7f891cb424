"""B200-native folded-VPP long-context prefill for a Qwen-style NVFP4 decoder.

Import name: ``qwen_infra_b200`` (registered by ``__graft_entry__.load_package``
or by installing the project).  Submodules:

* ``kernels``      torch-facing operators over the sm_100a C ABI
* ``vpp.layout``   folded placement and per-rank stage order for G ranks
* ``vpp.model``    virtual-stage layer compute (weights, paged NVFP4 KV)
* ``vpp.runner``   bank driver: one process per GPU, stage boundaries
* ``vpp.stages``   stage-boundary transport (P2P copy engine / NCCL)
* ``cli``          ``qwen-infra prefill`` command surface
"""

__all__ = ["kernels", "vpp"]
