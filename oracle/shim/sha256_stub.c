/* Stand-in for speech-mac src/sha256.c (CommonCrypto) in the oracle/_ref build.
 *
 * TEST INFRASTRUCTURE ONLY. The oracle never opens a .kpack: weights are
 * synthetic and handed to the reference as PhononTensorView structs. Pack
 * hash pinning (src/phonon_pack.c:72,155) is therefore unreachable; the stub
 * reports failure so that an accidental pack open fails loudly. */
#include <stddef.h>

int speech_sha256_hex(const unsigned char *data, size_t length, char output[65]);

int speech_sha256_hex(const unsigned char *data, size_t length, char output[65]) {
    (void)data;
    (void)length;
    if (output)
        output[0] = '\0';
    return 0;
}
