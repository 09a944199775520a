/* Links the C-ABI through the CMake package and checks host-side behaviour
 * (no GPU needed): version, status names and an argument error. */
#include <stdio.h>
#include <string.h>

#include "fkc_capi.h"

int main(void) {
  if (fkc_abi_version() != 1) return 1;
  if (strcmp(fkc_status_string(FKC_EWORKSPACE), "FKC_EWORKSPACE") != 0) return 2;
  if (fkc_assign(NULL, NULL, NULL, NULL, NULL, 1, 8, 2, 16, FKC_DTYPE_F16, NULL, 0, NULL) !=
      FKC_EINVAL)
    return 3;
  printf("capi consumer ok: %s\n", fkc_last_error());
  return 0;
}
