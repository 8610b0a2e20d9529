/* A plain C caller of the fgt C ABI (include/fgt.h), as the reference's
 * native executor would be: build a partition descriptor for a row softmax
 * (x - max, exp, / sum) over f32 [rows, cols], create the spec, read its
 * info, ports and Execution Plan, and check that invalid descriptors come
 * back as statuses with a message. Planning and sm_100a specialisation run
 * without a GPU; no launch is made. Prints "ok" and exits 0 on success. */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "fgt.h"

static fgt_node node(int32_t op, int32_t dt, int32_t rank, const int64_t* shape) {
  fgt_node n;
  memset(&n, 0, sizeof n);
  n.opcode = op;
  n.dtype = dt;
  n.rank = rank;
  for (int k = 0; k < rank; ++k) n.shape[k] = shape[k];
  return n;
}

static int fail(const char* what) {
  fprintf(stderr, "%s: %s\n", what, fgt_last_error());
  return 1;
}

int main(void) {
  if (fgt_abi_version() != FGT_ABI_VERSION) return fail("abi version");
  const int64_t rows = 64, cols = 1024;
  const int64_t rc[2] = {rows, cols}, r1[2] = {rows, 1}, r[1] = {rows};
  fgt_node nodes[8];
  nodes[0] = node(FGT_OP_PARAMETER, FGT_F32, 2, rc);
  nodes[0].num_attrs = 1;  /* input port 0 */
  nodes[1] = node(FGT_OP_REDUCE_MAX, FGT_F32, 1, r);
  nodes[1].num_operands = 1, nodes[1].operands[0] = 0, nodes[1].num_attrs = 1, nodes[1].attrs[0] = 1;
  nodes[2] = node(FGT_OP_RESHAPE, FGT_F32, 2, r1);
  nodes[2].num_operands = 1, nodes[2].operands[0] = 1;
  nodes[3] = node(FGT_OP_BROADCAST_IN_DIM, FGT_F32, 2, rc);
  nodes[3].num_operands = 1, nodes[3].operands[0] = 2, nodes[3].num_attrs = 2, nodes[3].attrs[0] = 0, nodes[3].attrs[1] = 1;
  /* x - max is the reference's x + max * (-1); here the subtraction is spelled
   * with a splat of -1 and a multiply, then an add */
  const int64_t none[1] = {0};
  nodes[4] = node(FGT_OP_CONSTANT, FGT_F32, 0, none);
  nodes[4].constant_bits = 0xbf800000u; /* -1.0f */
  nodes[5] = node(FGT_OP_SPLAT, FGT_F32, 2, rc);
  nodes[5].num_operands = 1, nodes[5].operands[0] = 4;
  nodes[6] = node(FGT_OP_MUL, FGT_F32, 2, rc);
  nodes[6].num_operands = 2, nodes[6].operands[0] = 3, nodes[6].operands[1] = 5;
  nodes[7] = node(FGT_OP_ADD, FGT_F32, 2, rc);
  nodes[7].num_operands = 2, nodes[7].operands[0] = 0, nodes[7].operands[1] = 6;
  int32_t outputs[1] = {7};
  fgt_partition_desc desc = {FGT_ABI_VERSION, 8, nodes, 1, outputs};

  fgt_spec* spec = NULL;
  if (fgt_spec_create(&desc, NULL, &spec) != FGT_OK) return fail("fgt_spec_create");
  fgt_spec_info info;
  if (fgt_spec_get_info(spec, &info) != FGT_OK) return fail("fgt_spec_get_info");
  if (info.num_inputs != 1 || info.num_outputs != 1 || info.kernel_count != 1) {
    fprintf(stderr, "unexpected info %d %d %d\n", info.num_inputs, info.num_outputs, info.kernel_count);
    return 1;
  }
  int32_t dt = -1, rank = -1;
  int64_t shape[FGT_MAX_RANK];
  if (fgt_spec_port(spec, 1, 0, &dt, &rank, shape) != FGT_OK) return fail("fgt_spec_port");
  if (dt != FGT_F32 || rank != 2 || shape[0] != rows || shape[1] != cols) return fail("output port");
  size_t need = 0;
  if (fgt_spec_plan_json(spec, NULL, 0, &need) != FGT_OK || need == 0) return fail("plan size");
  char* plan = (char*)malloc(need);
  if (fgt_spec_plan_json(spec, plan, need, &need) != FGT_OK) return fail("plan json");
  if (!strstr(plan, "\"schema_version\":1") || !strstr(plan, "cuda_lowering")) {
    fprintf(stderr, "plan: %.200s\n", plan);
    return 1;
  }
  free(plan);
  /* a launch with NULL buffers is rejected before anything runs */
  const void* in[1] = {NULL};
  void* out[1] = {NULL};
  if (fgt_spec_launch(spec, in, out, NULL, 0, NULL) == FGT_OK) return fail("NULL launch accepted");
  fgt_spec_destroy(spec);

  /* an invalid descriptor: the add's declared shape disagrees with its operands */
  nodes[7].shape[1] = cols + 1;
  spec = NULL;
  fgt_status st = fgt_spec_create(&desc, NULL, &spec);
  if (st != FGT_ERR_INVALID || spec != NULL || strlen(fgt_last_error()) == 0) {
    fprintf(stderr, "invalid descriptor accepted (status %d)\n", st);
    return 1;
  }
  printf("ok\n");
  return 0;
}
