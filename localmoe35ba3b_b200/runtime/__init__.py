"""Runtime around the operators.

* ``gpu_routes`` -- routing plan and the fused prefill MoE block (``moe_block``,
  ``routed_moe``);
* ``decode`` -- the one-token decode chain (``decode_block``);
* ``block`` -- the device router and the whole sparse-MoE block (``TopKRouter``,
  ``SparseMoeBlock``);
* ``checkpoint`` -- the converted-checkpoint loader (``load_blocks``);
* ``install`` -- ``install(model)``: swap a loaded model's blocks and INT8 linears;
* ``ep`` -- expert parallelism over ``torch.distributed`` (``moe_forward``).
"""
