"""vq2_vllm (B200): the vq2 routed-expert MoE path as a drop-in for the reference plugin."""
