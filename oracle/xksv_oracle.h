/* xksv_oracle.h -- TEST INFRASTRUCTURE ONLY: CPU restatement of the reference
 * slab codec (see xksv_oracle.c).  Same argument meaning and return codes as
 * the reference CPU ABI (src/c_api.cpp:17-85): 0 on success, -1 on error,
 * outputs malloc'd and released with oracle_free. */
#ifndef XKSV_ORACLE_H
#define XKSV_ORACLE_H
#include <stddef.h>
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif
int oracle_pack(const void* data, size_t n, size_t rows, size_t cols, void** out, size_t* out_size);
int oracle_unpack(const void* data, size_t n, size_t rows, size_t cols, void** out, size_t* out_size);
int oracle_pack_parallel(const void* data, size_t n, size_t rows, size_t cols, void** out, size_t* out_size);
int oracle_unpack_parallel(const void* data, size_t n, void** out, size_t* out_size);
int oracle_decode_into(const void* data, size_t n, size_t rows, size_t cols, int codec, void* dst);
void oracle_tile(const uint16_t* in, uint16_t* out, size_t rows, size_t cols);
void oracle_untile(const uint16_t* in, uint16_t* out, size_t rows, size_t cols);
void oracle_free(void* p);
#ifdef __cplusplus
}
#endif
#endif
