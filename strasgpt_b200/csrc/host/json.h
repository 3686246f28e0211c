// Minimal JSON document reader for the model directory files (config.json,
// model.safetensors.index.json, safetensors headers, tokenizer.json).
//
// Strings are kept RAW: the bytes between the quotes, escapes untouched.
// That is what the reference's scanner hands to its grammar
// (source/json_scanner.l:223-228), and the tokenizer depends on it.
#ifndef STRASGPT_JSON_H
#define STRASGPT_JSON_H

#include <stdbool.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  JSON_NULL,
  JSON_BOOL,
  JSON_NUMBER,
  JSON_STRING,
  JSON_ARRAY,
  JSON_OBJECT
} json_kind_t;

typedef struct json_value {
  json_kind_t kind;
  bool boolean;       // JSON_BOOL
  bool is_int;        // JSON_NUMBER: the literal is (or equals) an integer
  long long ival;     // JSON_NUMBER: valid when is_int
  double fval;        // JSON_NUMBER: always set
  char* string;       // JSON_STRING: raw bytes, NUL-terminated
  size_t count;       // JSON_ARRAY / JSON_OBJECT: number of children
  char** key;         // JSON_OBJECT: raw member names
  struct json_value* item; // children
  size_t line;        // line of the value's first character (1-based)
} json_value_t;

// Parse the first JSON value of text[0..len). Trailing bytes after it are
// ignored (safetensors headers are space-padded). Dies on a syntax error,
// naming `what` and the line.
json_value_t* json_parse(const char* text, size_t len, const char* what);

// Read a whole file and parse it. Returns NULL if the file cannot be opened.
json_value_t* json_parse_file(const char* path);

void json_free(json_value_t* v);

// Object member lookup (first match), NULL if absent or v is not an object.
const json_value_t* json_get(const json_value_t* v, const char* key);

#ifdef __cplusplus
}
#endif

#endif // STRASGPT_JSON_H
