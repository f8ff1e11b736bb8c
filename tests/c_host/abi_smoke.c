/* A C host binding libh3b through include/h3b.h alone (no Python, no torch):
 * prints the ABI version and checks that a call with a NULL pointer is
 * rejected on the host with H3B_ERR_ARG and a message -- the error behaviour a
 * C/FFI caller relies on.  Makes no device call, so it runs without a GPU. */
#include <stdio.h>
#include <string.h>

#include "h3b.h"

int main(void) {
    printf("abi %d\n", h3b_abi_version());
    int rc = h3b_quant_rowwise(NULL, 64, 4, 64, NULL, NULL, NULL);
    const char *msg = h3b_last_error();
    printf("rc %d\n", rc);
    printf("msg %s\n", msg ? msg : "(null)");
    return (rc == H3B_ERR_ARG && msg && strstr(msg, "h3b_quant_rowwise")) ? 0 : 1;
}
