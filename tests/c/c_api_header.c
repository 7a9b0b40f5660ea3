/* The C ABI header from a plain C11 translation unit: it must compile without
 * C++ (-std=c11 -pedantic -Wall -Wextra -Werror), link against the library and
 * answer calls that need no GPU, as tests/test_c_api_header.c checks the
 * reference's own header (include/voxcpm2/c_api.h). */
#include "voxcpm2_cuda.h"

#include <stdio.h>

int main(void) {
    vxc_model_desc desc = {0};
    vxc_stream* stream = NULL;
    vxc_stream_state state;
    int32_t status;

    if (vxc_abi_version() != VXC_ABI_VERSION) {
        fprintf(stderr, "abi version %u, header %u\n", vxc_abi_version(), VXC_ABI_VERSION);
        return 1;
    }
    /* null handles are invalid arguments, with a message */
    status = vxc_stream_create(NULL, 16, &stream);
    if (status != VXC_STATUS_INVALID_ARGUMENT || stream != NULL || vxc_last_error()[0] == '\0') return 2;
    status = vxc_read_state(NULL, &state);
    if (status != VXC_STATUS_INVALID_ARGUMENT) return 3;
    /* weight counts need no device: a zeroed description is rejected with 0 */
    if (vxc_component_weight_count(&desc, VXC_BASE_DECODER) != 0) return 4;
    vxc_device_destroy(NULL);
    vxc_stream_destroy(NULL);
    vxc_group_destroy(NULL);
    printf("ok %u\n", vxc_abi_version());
    return 0;
}
