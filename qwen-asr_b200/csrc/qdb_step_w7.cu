// qdb_step_w7.cu - second build of the persistent decode step: 7 consumer
// warps and 12 KB ring stages. Measured faster than the 6-warp / 16 KB build
// for hidden 1024 (row items of 6 rows), slower for hidden 2048, where 12 KB
// stages hold an odd 3 rows of K = 2048.
#define QDB_NCW 7
#define QDB_STAGE_BYTES 12288
#define QDB_STEP_ENTRY qdb_step_kernel_w7
#define QDB_STEP_NAME "w7s12"
#define QDB_STEP_COMMON 0
#include "qdb_step.cu"
