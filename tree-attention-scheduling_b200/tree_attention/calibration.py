"""B200 re-calibration of the scheduler's cost model.

Initial constants; replaced by the fitted values once calibrated on the GPU.
"""

B200_CONSTANTS = dict(
    bandwidth=6_000_000.0,
    cube_flops=1_200_000_000.0,
    task_us=0.02,
    merge_us=0.002,
    cube_rows=16,
    key_tile=256,
    kv_split=1024,
    max_query_rows=512,
)
