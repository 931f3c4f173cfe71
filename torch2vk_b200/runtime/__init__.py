"""B200 runtime surface mirroring torch2vk.runtime: LogicalTensor binding, shader contracts,
RuntimeSession (request / frame / dispatch / readback) and the CUDA op table behind dispatch."""
