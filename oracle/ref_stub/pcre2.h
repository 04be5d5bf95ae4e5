/* Declarations-only stand-in for the PCRE2 development header, which this
 * image lacks (only the runtime libpcre2-8.so.0 is installed).  It declares
 * just the 8-bit API the reference's tokenizer names, so the reference's
 * inferencer.cu compiles unmodified inside oracle/ref_harness.cu; the harness
 * never runs the tokenizer.  Names and signatures follow PCRE2's public API. */
#ifndef IJB_PCRE2_STUB_H
#define IJB_PCRE2_STUB_H
#include <stddef.h>
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif
typedef size_t PCRE2_SIZE;
typedef const uint8_t *PCRE2_SPTR8;
typedef struct pcre2_real_code_8 pcre2_code_8;
typedef struct pcre2_real_match_data_8 pcre2_match_data_8;
typedef struct pcre2_real_general_context_8 pcre2_general_context_8;
typedef struct pcre2_real_compile_context_8 pcre2_compile_context_8;
typedef struct pcre2_real_match_context_8 pcre2_match_context_8;
#define PCRE2_ZERO_TERMINATED (~(PCRE2_SIZE)0)
#define PCRE2_UCP 0x00020000u
#define PCRE2_UTF 0x00080000u
pcre2_code_8 *pcre2_compile_8(PCRE2_SPTR8, PCRE2_SIZE, uint32_t, int *, PCRE2_SIZE *, pcre2_compile_context_8 *);
void pcre2_code_free_8(pcre2_code_8 *);
pcre2_match_data_8 *pcre2_match_data_create_from_pattern_8(const pcre2_code_8 *, pcre2_general_context_8 *);
int pcre2_match_8(const pcre2_code_8 *, PCRE2_SPTR8, PCRE2_SIZE, PCRE2_SIZE, uint32_t, pcre2_match_data_8 *,
                  pcre2_match_context_8 *);
PCRE2_SIZE *pcre2_get_ovector_pointer_8(pcre2_match_data_8 *);
void pcre2_match_data_free_8(pcre2_match_data_8 *);
#ifdef __cplusplus
}
#endif
#define PCRE2_SPTR PCRE2_SPTR8
#define pcre2_code pcre2_code_8
#define pcre2_match_data pcre2_match_data_8
#define pcre2_compile pcre2_compile_8
#define pcre2_code_free pcre2_code_free_8
#define pcre2_match_data_create_from_pattern pcre2_match_data_create_from_pattern_8
#define pcre2_match pcre2_match_8
#define pcre2_get_ovector_pointer pcre2_get_ovector_pointer_8
#define pcre2_match_data_free pcre2_match_data_free_8
#endif
