// The reference's tokenizer.h calls through include/qwen_model_b200.h:
//     shim_tokenizer <model_dir> <text>   -> the token ids, one per line, then
//                                            "#" and the decoded text
#include <cstdio>
#include <string>
#include <vector>

#include "qwen_model_b200.h"

int main(int argc, char** argv) {
    if (argc != 3) { fprintf(stderr, "usage: shim_tokenizer <model_dir> <text>\n"); return 2; }
    Tokenizer t;
    build_tokenizer(&t, argv[1], 0);
    std::vector<int> ids(std::string(argv[2]).size() + 1);
    int n = 0;
    encode(&t, argv[2], ids.data(), &n);
    std::string back;
    for (int i = 0; i < n; i++) {
        printf("%d\n", ids[i]);
        back += decode(&t, ids[i]);
    }
    printf("#%s\n", back.c_str());
    free_tokenizer(&t);
    return 0;
}
