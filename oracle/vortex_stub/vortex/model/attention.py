"""Flash-attention kvcache entry point is absent here: the reference's driver
then treats attention as the slow path (evspark/specdec/block/driver.py:80-93)."""

local_flash_attn_with_kvcache = None
